// C ABI of the DF-SSM B200 decode engine: .dfssm loading, device arena, state,
// step execution (CUDA graph of per-op kernels, or the persistent step kernel) and the
// stand-alone reference-op replacements.  See include/dfssm.h for the contract.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "engine.h"
#include "kernels.cuh"
#include "sample.cuh"
#include "prefill.cuh"
#include "umma.cuh"

using namespace dfssm;

thread_local std::string g_err;

int dfssm_fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

namespace {

#define CU(call)                                                                              \
  do {                                                                                        \
    cudaError_t _e = (call);                                                                  \
    if (_e != cudaSuccess)                                                                    \
      return dfssm_fail(DFSSM_ERR_CUDA, "%s failed: %s (%d) at %s:%d", #call, cudaGetErrorString(_e), \
                  (int)_e, __FILE__, __LINE__);                                               \
  } while (0)

#define CHECK_LAUNCH() CU(cudaGetLastError())

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (device, kernel, size): the call costs
// microseconds of host time, which the stand-alone ops would otherwise pay on every launch.
cudaError_t ensure_smem(const void* fn, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, size_t> done;
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return ce;
  std::lock_guard<std::mutex> lk(mu);
  size_t& have = done[{dev, fn}];
  if (have >= bytes) return cudaSuccess;
  ce = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (ce == cudaSuccess) have = bytes;
  return ce;
}

constexpr size_t kHeader = 64;
constexpr int kRank = DFSSM_RANK;

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Layout {  // offsets inside the .dfssm image
  size_t emb, emb_s, layer0, layer_bytes, norm_f, total;
  size_t proj_bytes(int n, int k) const {
    return (size_t)n * (k / 32) * 4 + n * 2 + (size_t)n * kRank + n * 2 + (size_t)kRank * k + kRank * 2;
  }
};

}  // namespace


namespace {

// Automatic mode: the persistent whole-step kernel where it supports the batch and dims
// (batch <= 2), else the per-op kernels replayed from a CUDA graph.
// Makes the engine stream wait for the caller's stream `us` and, when the engine's earlier work was
// last ordered into another caller stream (where persistent steps may have run directly), for that
// stream too.
cudaError_t engine_stream_after(dfssm_engine* e, cudaStream_t us) {
  cudaError_t ce;
  if (e->order_valid && e->order_s != us) {
    if ((ce = cudaEventRecord(e->ev_cat, e->order_s)) != cudaSuccess) return ce;
    if ((ce = cudaStreamWaitEvent(e->s, e->ev_cat, 0)) != cudaSuccess) return ce;
  }
  if ((ce = cudaEventRecord(e->ev_in, us)) != cudaSuccess) return ce;
  return cudaStreamWaitEvent(e->s, e->ev_in, 0);
}

int effective_mode(const dfssm_engine* e) {
  if (e->mode != 0) return e->mode;
  // measured at the 1.3B shape: batches 1, 2 and 4 run one persistent launch (0.55, 0.72 and
  // 1.23 ms per step), batch 3 two (1.26 ms); from batch 5 the per-op graph on the mma.sync
  // projections is faster (1.76 ms at 5, 1.83 at 6 against 1.77 and 1.96 for two launches)
  static const int persist_max = [] {
    const char* v = getenv("DFSSM_PERSIST_MAX");
    return v ? atoi(v) : 4;
  }();
  return e->batch <= persist_max && persistent_supported(e) ? 3 : 1;
}

// ------------------------------------------------------------------ kernel launches

// A group is a contiguous range of the batch's sequences [b0, b0 + nb); every per-op kernel works
// on one group through row offsets of the batch-major buffers.
struct Group {
  int b0, nb;
};

// Outputs of the quantising prologue for a set of activation rows (row r at offset r).
struct RowBufs {
  __half* xn;
  int8_t* q;
  __half* xs;
  int* qsum;
  __half* t;
};
RowBufs engine_rows(dfssm_engine* e) { return RowBufs{e->xn, e->q, e->xs, e->qsum, e->t}; }

int launch_prep(dfssm_engine* e, const __half* in, int K, const float* w, int quant, const ProjW* p,
                cudaStream_t s, Group G, const RowBufs& R) {
  if (quant && p && K % 512 == 0) {
    const int kpt = K / 512;
    // rank parts per row: 8 while rows x 8 CTAs still fit on the SMs (measured at the 1.3B shape: batch 8
    // 1.59 -> 1.53 ms per step), else 2 (4 parts were 2% slower at batches 32 and 64); DFSSM_PREP_PARTS
    // overrides
    static const int force_parts = [] {
      const char* v = getenv("DFSSM_PREP_PARTS");
      return v ? atoi(v) : 0;
    }();
    const int parts = force_parts ? force_parts : (G.nb * 8 <= e->sm_count ? 8 : 2);
#define DFSSM_PREP_FAST_P(n, P)                                                                             \
  if (kpt == n && parts == P) {                                                                             \
    act_prep_fast_kernel<n, P><<<dim3(G.nb, P), kPrepFastThreads, 0, s>>>(in + (size_t)G.b0 * K, K, w,      \
        R.q + (size_t)G.b0 * K, R.xs + G.b0, R.qsum + G.b0, p->B16, R.t + G.b0 * kRank);                    \
    CHECK_LAUNCH();                                                                                        \
    return DFSSM_OK;                                                                                       \
  }
#define DFSSM_PREP_FAST(n) DFSSM_PREP_FAST_P(n, 2) DFSSM_PREP_FAST_P(n, 4) DFSSM_PREP_FAST_P(n, 8)
    DFSSM_PREP_FAST(1)
    DFSSM_PREP_FAST(2)
    DFSSM_PREP_FAST(4)
    DFSSM_PREP_FAST(8)
    DFSSM_PREP_FAST(5)
    DFSSM_PREP_FAST(10)
#undef DFSSM_PREP_FAST
#undef DFSSM_PREP_FAST_P
  }
  const size_t sm = (size_t)K * sizeof(__half);
  act_prep_kernel<<<G.nb, kPrepThreads, sm, s>>>(in + (size_t)G.b0 * K, K, w, quant, R.xn + (size_t)G.b0 * K,
                                                 R.q + (size_t)G.b0 * K, R.xs + G.b0, R.qsum + G.b0,
                                                 p ? p->B16 : nullptr, R.t + G.b0 * kRank);
  CHECK_LAUNCH();
  return DFSSM_OK;
}

int gemv_grid(const dfssm_engine* e, int N) {
  const int rows_per_cta = 2 * (kGemvThreads / 32);
  int g = (N + rows_per_cta - 1) / rows_per_cta;
  return g < 1 ? 1 : g;
}

// Tensor-core projection for batches of 8 or more: RG row groups of 16 per CTA (2 for the wide
// in_proj, 1 for out_proj so that enough CTAs exist), K split over the remaining warps.
constexpr int kMmaMinBatch = 8;
inline bool mma_ok(int K, int RG) {
  const int KS = (kMmaThreads / 32) / RG;
  return K % 128 == 0 && ((K / 32) % KS) == 0 && ((K / 32 / KS) % 4) == 0 && (K / 32 / KS) <= 4 * kMmaMaxBlk;
}
// Batch from which the engine's per-op projections use the mma.sync kernel instead of the 1-bit
// GEMV (DFSSM_MMA_MIN overrides it): at the 1.3B shape the per-op step took 1.60 ms at batch 3 on
// mma.sync against ~2.8 ms on the GEMV.
int mma_min_batch() {
  static const int v = [] {
    const char* e = getenv("DFSSM_MMA_MIN");
    return e ? atoi(e) : 3;
  }();
  return v;
}
// Row groups per CTA for an N x K projection (0 = no tensor-core configuration fits).
inline int mma_rg(int N, int K) {
  const int pref = N >= 4096 ? 2 : 1, other = 3 - pref;
  return mma_ok(K, pref) ? pref : (mma_ok(K, other) ? other : 0);
}


// Split-K scratch of the tcgen05 projection: int32 partial sums [rows][N] and one counter per
// output tile, all zero between uses (the kernel clears what it used).
struct UmmaScratch {
  int* acc = nullptr;
  unsigned* cnt = nullptr;
};
constexpr int kUmmaMaxTiles = 4096;

// Batch at and above which the projections use the tcgen05 kernel (DFSSM_UMMA_MIN overrides).
int umma_min_batch() {
  static const int v = [] {
    const char* e = getenv("DFSSM_UMMA_MIN");
    return e ? atoi(e) : kUmmaMinBatch;
  }();
  return v;
}

// Device address of g_umma_err on the current device (looked up once per device).
cudaError_t umma_err_word(unsigned** out) {
  static std::mutex mu;
  static std::map<int, unsigned*> addr;
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return ce;
  std::lock_guard<std::mutex> lk(mu);
  auto it = addr.find(dev);
  if (it == addr.end()) {
    unsigned* a = nullptr;
    ce = cudaGetSymbolAddress(reinterpret_cast<void**>(&a), g_umma_err);
    if (ce != cudaSuccess) return ce;
    it = addr.emplace(dev, a).first;
  }
  *out = it->second;
  return cudaSuccess;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link); null if absent.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    cudaGetLastError();
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

// Tensor map over the activation rows q [rows][K] int8: box 128 bytes x NT rows, 128-byte swizzle,
// rows past `rows` read as zeros.  False if it cannot be made.
bool make_q_map(CUtensorMap* m, const int8_t* q, int rows, int K, int NT) {
  const EncodeTiledFn fn = encode_tiled();
  if (!fn || (reinterpret_cast<uintptr_t>(q) & 15) || K % 128) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K};
  const cuuint32_t box[2] = {128u, (cuuint32_t)NT};
  const cuuint32_t estr[2] = {1u, 1u};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(q), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Returns -1 (nothing launched) when the tcgen05 kernel cannot take this call: no tensor map (the
// driver entry point is missing, or misaligned operands); the caller then uses the mma.sync kernel.
// Tensor map over packed 1-bit weights [N rows][K / 8 bytes]: box 16 bytes x 128 rows, no swizzle,
// rows past N read as zeros.
bool make_w_map(CUtensorMap* m, const uint32_t* bits, int N, int K) {
  const EncodeTiledFn fn = encode_tiled();
  if (!fn || (reinterpret_cast<uintptr_t>(bits) & 15) || K % 128) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)(K / 8), (cuuint64_t)N};
  const cuuint64_t strides[1] = {(cuuint64_t)(K / 8)};
  const cuuint32_t box[2] = {16u, 128u};
  const cuuint32_t estr[2] = {1u, 1u};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint32_t*>(bits), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MODE, int NT>
int launch_umma(const ProjW& p, int B, const int8_t* q, const int* qsum, const __half* xs, const __half* t, void* out,
                int ld_out, float* conv_state, const __half* conv_w, const __half* conv_b, int d_inner, int d_xbc,
                cudaStream_t s, UmmaScratch us) {
  const int tiles = ((p.N + 127) / 128) * ((B + NT - 1) / NT);
  // split K until about one CTA per SM: MODE 2 adds the partials into `out`, the others need the
  // scratch
  int ks = 1;
  const bool can_split = MODE == 2 || (us.acc && us.cnt && tiles <= kUmmaMaxTiles);
  static const int target = [] {
    const char* e = getenv("DFSSM_UMMA_CTAS");
    return e ? atoi(e) : 160;
  }();
  while (can_split && tiles * ks * 2 <= target && (p.K / (2 * ks)) % kUmmaKC == 0 && ks < 16) ks *= 2;
  const size_t sm = proj_umma_smem(NT);
  CUtensorMap tm, tw;
  memset(&tm, 0, sizeof(tm));
  memset(&tw, 0, sizeof(tw));
  if (!make_q_map(&tm, q, B, p.K, NT) || !make_w_map(&tw, p.bits, p.N, p.K)) return -1;
  if (MODE == 2 && ks > 1) CU(cudaMemsetAsync(out, 0, (size_t)B * ld_out * 4, s));
  unsigned* err = nullptr;
  CU(umma_err_word(&err));
  const dim3 grid((p.N + 127) / 128, (B + NT - 1) / NT, ks);
  CU(ensure_smem(reinterpret_cast<const void*>(proj_umma_kernel<MODE, NT>), sm));
  proj_umma_kernel<MODE, NT><<<grid, kUmmaThreads, sm, s>>>(tm, tw, p, qsum, xs, t, B, reinterpret_cast<__half*>(out),
                                                             ld_out, conv_state, conv_w, conv_b, d_inner, d_xbc, ks,
                                                             us.acc, us.cnt, err);
  CHECK_LAUNCH();
  return DFSSM_OK;
}

template <int MODE>
int launch_mma(const ProjW& p, int B, const int8_t* q, const int* qsum, const __half* xs, const __half* t, void* out,
               int ld_out, float* conv_state, const __half* conv_w, const __half* conv_b, int d_inner, int d_xbc,
               cudaStream_t s, UmmaScratch us = UmmaScratch{}) {
  if (B >= umma_min_batch() && p.K % kUmmaKC == 0) {  // tcgen05 path
    // the widest batch tile that still gives enough tiles to fill the GPU without splitting K: a
    // split leaves the epilogue to the last CTA of each tile
    static const int min_tiles = [] {
      const char* e = getenv("DFSSM_UMMA_TILES");
      return e ? atoi(e) : 120;
    }();
    auto tiles = [&](int nt) { return ((p.N + 127) / 128) * ((B + nt - 1) / nt); };
    int NT = B >= 128 ? 128 : (B >= 64 ? 64 : 32);
    while (NT > 32 && tiles(NT) < min_tiles) NT /= 2;
    const int rc = NT == 128 ? launch_umma<MODE, 128>(p, B, q, qsum, xs, t, out, ld_out, conv_state, conv_w, conv_b, d_inner, d_xbc, s, us)
                 : NT == 64  ? launch_umma<MODE, 64>(p, B, q, qsum, xs, t, out, ld_out, conv_state, conv_w, conv_b, d_inner, d_xbc, s, us)
                             : launch_umma<MODE, 32>(p, B, q, qsum, xs, t, out, ld_out, conv_state, conv_w, conv_b, d_inner, d_xbc, s, us);
    if (rc != -1) return rc;  // -1: not taken, fall through to mma.sync
  }
  const int RG = mma_rg(p.N, p.K);
  // batch tiles of 8 per pass: the fewest that hold the batch (batches above 32 run passes of 32)
  const int NT = B <= 8 ? 1 : B <= 16 ? 2 : 4;
  const size_t sm = proj_mma_smem(p.K, RG, NT);
#define DFSSM_MMA_LAUNCH(rg, nt)                                                                            \
  if (RG == rg && NT == nt) {                                                                               \
    CU(ensure_smem(reinterpret_cast<const void*>(proj_mma_kernel<MODE, rg, nt>), sm));                      \
    proj_mma_kernel<MODE, rg, nt><<<(p.N + 16 * rg - 1) / (16 * rg), kMmaThreads, sm, s>>>(                 \
        p, q, qsum, xs, t, B, reinterpret_cast<__half*>(out), ld_out, conv_state, conv_w, conv_b, d_inner, d_xbc); \
    CHECK_LAUNCH();                                                                                         \
    return DFSSM_OK;                                                                                        \
  }
  DFSSM_MMA_LAUNCH(2, 1) DFSSM_MMA_LAUNCH(2, 2) DFSSM_MMA_LAUNCH(2, 4)
  DFSSM_MMA_LAUNCH(1, 1) DFSSM_MMA_LAUNCH(1, 2) DFSSM_MMA_LAUNCH(1, 4)
#undef DFSSM_MMA_LAUNCH
  return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "no mma.sync projection instance for RG %d", RG);
}

template <int MODE>
int launch_gemv(dfssm_engine* e, const ProjW& p, int B, const int8_t* q, const int* qsum, const __half* xs,
                const __half* t, void* out, int ld_out, float* conv_state, const LayerW* L, cudaStream_t s,
                UmmaScratch us) {
  if (B >= mma_min_batch() && mma_rg(p.N, p.K))
    return launch_mma<MODE>(p, B, q, qsum, xs, t, out, ld_out, conv_state, L ? L->conv_w : nullptr,
                            L ? L->conv_b : nullptr, e->d.d_inner, e->d.d_xbc, s, us);
  const size_t sm = (size_t)kGemvBT * p.K;
  proj_gemv_kernel<MODE><<<gemv_grid(e, p.N), kGemvThreads, sm, s>>>(
      p, q, qsum, xs, t, B, reinterpret_cast<__half*>(out), ld_out, conv_state, L ? L->conv_w : nullptr,
      L ? L->conv_b : nullptr, e->d.d_inner, e->d.d_xbc);
  CHECK_LAUNCH();
  return DFSSM_OK;
}

int enqueue_layer(dfssm_engine* e, int l, cudaStream_t s, Group G) {
  const dfssm_dims& d = e->d;
  const LayerW& L = e->layers[l];
  const int B = G.nb, b0 = G.b0;
  // the split-K scratch is shared: only a step that runs the whole batch as one group uses it
  const UmmaScratch us = (b0 == 0 && B == e->batch) ? UmmaScratch{e->uacc, e->ucnt} : UmmaScratch{};
  const size_t hd = (size_t)d.nheads * DFSSM_HEADDIM * DFSSM_DSTATE;
  int rc;
  if ((rc = launch_prep(e, e->x, d.d_model, L.ln_w, 1, &L.in, s, G, engine_rows(e)))) return rc;
  if ((rc = launch_gemv<0>(e, L.in, B, e->q + (size_t)b0 * d.d_model, e->qsum + b0, e->xs + b0, e->t + b0 * kRank,
                           e->proj + (size_t)b0 * d.n_in, d.n_in,
                           e->conv + (size_t)l * e->conv_layer + (size_t)b0 * 3 * d.d_xbc, &L, s, us)))
    return rc;
  __half* pr = e->proj + (size_t)b0 * d.n_in;
  ssm_gate_kernel<<<dim3(d.nheads, B), kSsmThreads, 0, s>>>(
      pr + d.d_inner, d.n_in, pr + d.d_inner + d.d_xbc, d.n_in, pr, d.n_in, d.d_inner, d.d_state, d.nheads,
      L.dt_bias, L.A_log, L.Dp, e->ssm + (size_t)l * e->ssm_layer + (size_t)b0 * hd,
      e->gated + (size_t)b0 * d.d_inner, d.d_inner);
  CHECK_LAUNCH();
  if ((rc = launch_prep(e, e->gated, d.d_inner, L.norm_w, 1, &L.out, s, G, engine_rows(e)))) return rc;
  if ((rc = launch_gemv<1>(e, L.out, B, e->q + (size_t)b0 * d.d_inner, e->qsum + b0, e->xs + b0, e->t + b0 * kRank,
                           e->x + (size_t)b0 * d.d_model, d.d_model, nullptr, nullptr, s, us)))
    return rc;
  return DFSSM_OK;
}

// Number of independent sequence groups the per-op step is split into.  Each group's layer chain is
// captured on its own stream, so the projection kernels of one group can overlap the state update
// of another.  Default 1; DFSSM_GROUPS=2..4 selects a split.
int step_groups(const dfssm_engine* e) {
  const char* env = getenv("DFSSM_GROUPS");
  if (env) {
    const int g = atoi(env);
    if (g >= 1 && g <= kMaxGroups && e->batch >= g) return g;
  }
  return 1;  // measured on B200 at batch 32: 2 groups 9% and 4 groups 28% slower than 1 (the
             // concurrent kernels compete for shared memory instead of filling idle time)
}

// The tensor-core LM head over `grid` CTAs with the fewest batch tiles of 8 per pass that hold B.
int launch_head_mma(const int8_t* Eq, const float* Es, int vocab, int d, const __half* xn, int B, float* logits,
                    unsigned long long* best, int grid, cudaStream_t s) {
  const int NT = B <= 8 ? 1 : B <= 16 ? 2 : 4;
  const size_t sm = lm_head_mma_smem(d, NT);
#define DFSSM_HEAD_LAUNCH(nt)                                                                                  \
  if (NT == nt) {                                                                                              \
    CU(ensure_smem(reinterpret_cast<const void*>(lm_head_mma_kernel<nt>), sm));                                \
    lm_head_mma_kernel<nt><<<grid, kHeadMmaThreads, sm, s>>>(Eq, Es, vocab, d, xn, B, logits, best);           \
    CHECK_LAUNCH();                                                                                            \
    return DFSSM_OK;                                                                                           \
  }
  DFSSM_HEAD_LAUNCH(1) DFSSM_HEAD_LAUNCH(2) DFSSM_HEAD_LAUNCH(4)
#undef DFSSM_HEAD_LAUNCH
  return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "no LM-head instance for %d batch tiles", NT);
}

int enqueue_head(dfssm_engine* e, cudaStream_t s) {
  const dfssm_dims& d = e->d;
  int rc;
  if ((rc = launch_prep(e, e->x, d.d_model, e->norm_f, 0, nullptr, s, Group{0, e->batch}, engine_rows(e)))) return rc;
  // the tensor-core head from batch 3 (DFSSM_HEAD_MMA_MIN overrides): at the 1.3B shape the
  // per-row GEMV head cost batches 5-7 about 0.25 ms more per step than batch 8 on the MMA head
  static const int head_mma_min = [] {
    const char* v = getenv("DFSSM_HEAD_MMA_MIN");
    return v ? atoi(v) : 3;
  }();
  if (e->batch >= head_mma_min && d.d_model % (64 * kHeadMmaU) == 0) {
    int rc2 = launch_head_mma(e->Eq, e->Es, d.vocab, d.d_model, e->xn, e->batch, e->logits, e->best, e->sm_count, s);
    if (rc2) return rc2;
  } else {
    const size_t sm = (size_t)kHeadBT * d.d_model * sizeof(float);
    lm_head_kernel<<<e->sm_count * 4, kHeadThreads, sm, s>>>(e->Eq, e->Es, d.vocab, d.d_model, e->xn, e->batch,
                                                             e->logits, e->best);
  }
  CHECK_LAUNCH();
  finalize_kernel<<<(e->batch + 127) / 128, 128, 0, s>>>(e->best, e->batch, e->tokens);
  CHECK_LAUNCH();
  return DFSSM_OK;
}

int enqueue_step_ops(dfssm_engine* e, cudaStream_t s) {
  const dfssm_dims& d = e->d;
  embed_kernel<<<e->batch, 256, 0, s>>>(e->tokens, e->Eq, e->Es, d.d_model, d.vocab, e->x);
  CHECK_LAUNCH();
  int rc;
  const int G = step_groups(e);
  if (G == 1) {
    for (int l = 0; l < d.n_layer; ++l)
      if ((rc = enqueue_layer(e, l, s, Group{0, e->batch}))) return rc;
    return enqueue_head(e, s);
  }
  // fork: group g runs all layers on stream gs[g] (group 0 on s), then join before the LM head
  CU(cudaEventRecord(e->ev_fork, s));
  for (int g = 1; g < G; ++g) CU(cudaStreamWaitEvent(e->gs[g], e->ev_fork, 0));
  for (int g = 0; g < G; ++g) {
    const int b0 = (int)((long long)e->batch * g / G), b1 = (int)((long long)e->batch * (g + 1) / G);
    cudaStream_t gsg = g == 0 ? s : e->gs[g];
    for (int l = 0; l < d.n_layer; ++l)
      if ((rc = enqueue_layer(e, l, gsg, Group{b0, b1 - b0}))) return rc;
  }
  for (int g = 1; g < G; ++g) {
    CU(cudaEventRecord(e->ev_join[g], e->gs[g]));
    CU(cudaStreamWaitEvent(s, e->ev_join[g], 0));
  }
  return enqueue_head(e, s);
}

int enqueue_step(dfssm_engine* e, int mode, cudaStream_t s) {
  if (mode == 3) return launch_persistent_step(e, s);
  return enqueue_step_ops(e, s);
}

int ensure_graph(dfssm_engine* e, int mode) {
  if (e->gexec && e->graph_batch == e->batch && e->graph_mode == mode) return DFSSM_OK;
  if (e->gexec) {
    cudaGraphExecDestroy(e->gexec);
    e->gexec = nullptr;
  }
  cudaGraph_t g = nullptr;
  CU(cudaStreamBeginCapture(e->s, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_step(e, mode, e->s);
  cudaError_t ce = cudaStreamEndCapture(e->s, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (ce != cudaSuccess) return dfssm_fail(DFSSM_ERR_CUDA, "graph capture failed: %s", cudaGetErrorString(ce));
  ce = cudaGraphInstantiate(&e->gexec, g, 0);
  cudaGraphDestroy(g);
  if (ce != cudaSuccess) return dfssm_fail(DFSSM_ERR_CUDA, "graph instantiate failed: %s", cudaGetErrorString(ce));
  e->graph_batch = e->batch;
  e->graph_mode = mode;
  return DFSSM_OK;
}

// ------------------------------------------------------------------ loading

int parse_dims(const unsigned char* img, size_t n, dfssm_dims* d, int* emb_kind) {
  if (n < kHeader) return dfssm_fail(DFSSM_ERR_FORMAT, "image shorter than the 64-byte header (%zu bytes)", n);
  if (memcmp(img, "DFSSM001", 8) != 0) return dfssm_fail(DFSSM_ERR_FORMAT, "bad magic (expected DFSSM001)");
  uint32_t h[9];
  memcpy(h, img + 8, sizeof(h));
  d->n_layer = (int)h[0];
  d->d_model = (int)h[1];
  d->d_inner = (int)h[2];
  d->d_state = (int)h[3];
  d->nheads = (int)h[4];
  d->headdim = (int)h[5];
  d->ngroups = (int)h[6];
  d->vocab = (int)h[7];
  *emb_kind = img[8 + 36];
  if (d->n_layer <= 0 || d->n_layer > 4096 || d->d_model <= 0 || d->d_inner <= 0 || d->vocab <= 0 ||
      d->nheads <= 0 || d->d_model > (1 << 16) || d->d_inner > (1 << 16) || d->vocab > (1 << 24))
    return dfssm_fail(DFSSM_ERR_FORMAT, "implausible header dims");
  if ((int64_t)d->nheads * d->headdim != d->d_inner)
    return dfssm_fail(DFSSM_ERR_FORMAT, "nheads*headdim (%d*%d) != d_inner (%d)", d->nheads, d->headdim, d->d_inner);
  if (d->ngroups != 1) return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "ngroups=%d (only 1 supported)", d->ngroups);
  if (d->headdim != DFSSM_HEADDIM || d->d_state != DFSSM_DSTATE)
    return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "headdim=%d d_state=%d (kernels are built for 64/128)", d->headdim,
                d->d_state);
  if (d->d_model % 128 || d->d_inner % 128)
    return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "d_model and d_inner must be multiples of 128");
  if (*emb_kind != 0 && *emb_kind != 1) return dfssm_fail(DFSSM_ERR_FORMAT, "unknown embedding kind %d", *emb_kind);
  d->d_xbc = d->d_inner + 2 * d->ngroups * d->d_state;
  d->n_in = 2 * d->d_inner + 2 * d->ngroups * d->d_state + d->nheads;
  return DFSSM_OK;
}

// Device arena: per layer, each array starts on a 256-byte boundary.
struct ArenaPlan {
  struct P {
    size_t bits, scale, A16, B16;
  };
  struct Lyr {
    P in, out;
    size_t conv_w, conv_b, A_log, Dp, dt_bias, norm_w, ln_w;
  };
  std::vector<Lyr> L;
  size_t Eq, Es, norm_f, total;
};

ArenaPlan plan_arena(const dfssm_dims& d) {
  ArenaPlan a;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  auto proj = [&](int n, int k) {
    ArenaPlan::P p;
    p.bits = take((size_t)n * (k / 32) * 4);
    p.scale = take((size_t)n * 2);
    p.A16 = take((size_t)n * kRank * 2);
    p.B16 = take((size_t)kRank * k * 2);
    return p;
  };
  for (int l = 0; l < d.n_layer; ++l) {
    ArenaPlan::Lyr y;
    y.in = proj(d.n_in, d.d_model);
    y.out = proj(d.d_model, d.d_inner);
    y.conv_w = take((size_t)d.d_xbc * 4 * 2);
    y.conv_b = take((size_t)d.d_xbc * 2);
    y.A_log = take((size_t)d.nheads * 4);
    y.Dp = take((size_t)d.nheads * 4);
    y.dt_bias = take((size_t)d.nheads * 4);
    y.norm_w = take((size_t)d.d_inner * 4);
    y.ln_w = take((size_t)d.d_model * 4);
    a.L.push_back(y);
  }
  a.norm_f = take((size_t)d.d_model * 4);
  a.Es = take((size_t)d.vocab * 4);
  a.Eq = take((size_t)d.vocab * d.d_model);
  a.total = off;
  return a;
}

int build_engine(const unsigned char* img, size_t n, int device, int max_batch, dfssm_engine** out) {
  if (!out) return dfssm_fail(DFSSM_ERR_ARG, "out is NULL");
  *out = nullptr;
  if (!img) return dfssm_fail(DFSSM_ERR_ARG, "image is NULL");
  if (max_batch < 1 || max_batch > 4096) return dfssm_fail(DFSSM_ERR_ARG, "max_batch=%d out of range", max_batch);
  dfssm_dims d;
  int emb_kind = 0;
  int rc = parse_dims(img, n, &d, &emb_kind);
  if (rc) return rc;
  const size_t emb_bytes = emb_kind == 0 ? (size_t)d.vocab * d.d_model * 2 : (size_t)d.vocab * d.d_model + (size_t)d.vocab * 2;
  Layout lay;
  const size_t per_layer = lay.proj_bytes(d.n_in, d.d_model) + lay.proj_bytes(d.d_model, d.d_inner) +
                           (size_t)d.d_xbc * 4 * 2 + (size_t)d.d_xbc * 2 + 3 * (size_t)d.nheads * 4 +
                           (size_t)d.d_inner * 4 + (size_t)d.d_model * 4;
  const size_t need = kHeader + emb_bytes + (size_t)d.n_layer * per_layer + (size_t)d.d_model * 4;
  if (n != need) return dfssm_fail(DFSSM_ERR_FORMAT, "image is %zu bytes, header implies %zu", n, need);

  ArenaPlan ap = plan_arena(d);
  std::vector<char> host(ap.total, 0);
  size_t src = kHeader;
  auto copy = [&](size_t dst, size_t bytes) {
    memcpy(host.data() + dst, img + src, bytes);
    src += bytes;
  };
  // embedding: int8 rows + fp32 per-row scale
  {
    int8_t* Eq = reinterpret_cast<int8_t*>(host.data() + ap.Eq);
    float* Es = reinterpret_cast<float*>(host.data() + ap.Es);
    if (emb_kind == 1) {
      memcpy(Eq, img + src, (size_t)d.vocab * d.d_model);
      src += (size_t)d.vocab * d.d_model;
      const __half* hs = reinterpret_cast<const __half*>(img + src);
      for (int v = 0; v < d.vocab; ++v) Es[v] = __half2float(hs[v]);
      src += (size_t)d.vocab * 2;
    } else {
      // fp16 embedding: per-row symmetric int8 quantisation, scale = absmax / 127.
      const __half* E = reinterpret_cast<const __half*>(img + src);
      for (int v = 0; v < d.vocab; ++v) {
        const __half* row = E + (size_t)v * d.d_model;
        float amax = 0.f;
        for (int k = 0; k < d.d_model; ++k) amax = fmaxf(amax, fabsf(__half2float(row[k])));
        const float s = amax > 0.f ? amax / 127.0f : 1.0f;
        Es[v] = s;
        for (int k = 0; k < d.d_model; ++k) {
          float qv = nearbyintf(__half2float(row[k]) / s);
          qv = fminf(127.f, fmaxf(-127.f, qv));
          Eq[(size_t)v * d.d_model + k] = (int8_t)qv;
        }
      }
      src += (size_t)d.vocab * d.d_model * 2;
    }
  }
  for (int l = 0; l < d.n_layer; ++l) {
    const ArenaPlan::Lyr& y = ap.L[l];
    const ArenaPlan::P* ps[2] = {&y.in, &y.out};
    const int ns[2] = {d.n_in, d.d_model}, ks[2] = {d.d_model, d.d_inner};
    for (int j = 0; j < 2; ++j) {
      copy(ps[j]->bits, (size_t)ns[j] * (ks[j] / 32) * 4);
      copy(ps[j]->scale, (size_t)ns[j] * 2);
      // LoRA: int8 + fp16 scale on disk, dequantised to fp16 here exactly as the reference loader
      // does ((q.float() * s.float()).half(), df_ssm_inference.py:78-83,92-97)
      {
        const int8_t* Aq = reinterpret_cast<const int8_t*>(img + src);
        const __half* As = reinterpret_cast<const __half*>(img + src + (size_t)ns[j] * kRank);
        __half* A16 = reinterpret_cast<__half*>(host.data() + ps[j]->A16);
        for (size_t r = 0; r < (size_t)ns[j]; ++r)
          for (int c = 0; c < kRank; ++c) A16[r * kRank + c] = __float2half_rn((float)Aq[r * kRank + c] * __half2float(As[r]));
        src += (size_t)ns[j] * kRank + (size_t)ns[j] * 2;
        const int8_t* Bq = reinterpret_cast<const int8_t*>(img + src);
        const __half* Bs = reinterpret_cast<const __half*>(img + src + (size_t)kRank * ks[j]);
        __half* B16 = reinterpret_cast<__half*>(host.data() + ps[j]->B16);
        for (int r = 0; r < kRank; ++r)
          for (size_t c = 0; c < (size_t)ks[j]; ++c)
            B16[r * (size_t)ks[j] + c] = __float2half_rn((float)Bq[r * (size_t)ks[j] + c] * __half2float(Bs[r]));
        src += (size_t)kRank * ks[j] + kRank * 2;
      }
    }
    copy(y.conv_w, (size_t)d.d_xbc * 4 * 2);
    copy(y.conv_b, (size_t)d.d_xbc * 2);
    copy(y.A_log, (size_t)d.nheads * 4);
    copy(y.Dp, (size_t)d.nheads * 4);
    copy(y.dt_bias, (size_t)d.nheads * 4);
    copy(y.norm_w, (size_t)d.d_inner * 4);
    copy(y.ln_w, (size_t)d.d_model * 4);
  }
  copy(ap.norm_f, (size_t)d.d_model * 4);
  if (src != n) return dfssm_fail(DFSSM_ERR_FORMAT, "internal: parsed %zu of %zu bytes", src, n);

  dfssm_engine* e = new dfssm_engine();
  e->device = device;
  e->d = d;
  e->emb_kind = emb_kind;
  e->max_batch = max_batch;
  e->batch = max_batch;
  auto cleanup = [&](int code) {
    dfssm_destroy(e);
    return code;
  };
  cudaError_t ce = cudaSetDevice(device);
  if (ce != cudaSuccess) return cleanup(dfssm_fail(DFSSM_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(ce)));
  cudaDeviceGetAttribute(&e->sm_count, cudaDevAttrMultiProcessorCount, device);
  if (cudaMalloc(&e->arena, ap.total) != cudaSuccess)
    return cleanup(dfssm_fail(DFSSM_ERR_OOM, "cudaMalloc(%zu) for weights failed", ap.total));
  e->arena_bytes = ap.total;
  ce = cudaMemcpy(e->arena, host.data(), ap.total, cudaMemcpyHostToDevice);
  if (ce != cudaSuccess) return cleanup(dfssm_fail(DFSSM_ERR_CUDA, "weight upload: %s", cudaGetErrorString(ce)));
  char* A = e->arena;
  for (int l = 0; l < d.n_layer; ++l) {
    const ArenaPlan::Lyr& y = ap.L[l];
    LayerW L;
    auto mk = [&](const ArenaPlan::P& p, int nrows, int k) {
      ProjW w;
      w.bits = reinterpret_cast<const uint32_t*>(A + p.bits);
      w.scale = reinterpret_cast<const __half*>(A + p.scale);
      w.A16 = reinterpret_cast<const __half*>(A + p.A16);
      w.B16 = reinterpret_cast<const __half*>(A + p.B16);
      w.N = nrows;
      w.K = k;
      return w;
    };
    L.in = mk(y.in, d.n_in, d.d_model);
    L.out = mk(y.out, d.d_model, d.d_inner);
    L.conv_w = reinterpret_cast<const __half*>(A + y.conv_w);
    L.conv_b = reinterpret_cast<const __half*>(A + y.conv_b);
    L.A_log = reinterpret_cast<const float*>(A + y.A_log);
    L.Dp = reinterpret_cast<const float*>(A + y.Dp);
    L.dt_bias = reinterpret_cast<const float*>(A + y.dt_bias);
    L.norm_w = reinterpret_cast<const float*>(A + y.norm_w);
    L.ln_w = reinterpret_cast<const float*>(A + y.ln_w);
    e->layers.push_back(L);
  }
  e->Eq = reinterpret_cast<const int8_t*>(A + ap.Eq);
  e->Es = reinterpret_cast<const float*>(A + ap.Es);
  e->norm_f = reinterpret_cast<const float*>(A + ap.norm_f);

  // state + activations
  const int B = max_batch;
  const int kmax = d.d_inner > d.d_model ? d.d_inner : d.d_model;
  e->ssm_layer = (size_t)B * d.nheads * DFSSM_HEADDIM * DFSSM_DSTATE;
  e->conv_layer = (size_t)B * 3 * d.d_xbc;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  // The persistent kernel's sync words and tagged exchange words (x, B/C, gated and LoRA t for 2
  // layer parities x its largest launch group, in replicas) come first, at the allocation's
  // aligned base: their L2 placement affects every exchange, so it must not move with the batch
  // capacity or the model's state size.
  const size_t o_sync = take(4096);
  const size_t o_xch = take(persistent_xch_bytes(d));
  const size_t o_ssm = take(e->ssm_layer * d.n_layer * 4);
  const size_t o_conv = take(e->conv_layer * d.n_layer * 4);
  const size_t o_x = take((size_t)B * d.d_model * 2);
  const size_t o_xn = take((size_t)B * kmax * 2);
  const size_t o_q = take((size_t)B * kmax);
  const size_t o_xs = take((size_t)B * 2);
  const size_t o_qsum = take((size_t)B * 4);
  const size_t o_t = take((size_t)B * kRank * 2);
  const size_t o_proj = take((size_t)B * d.n_in * 2);
  const size_t o_gated = take((size_t)B * d.d_inner * 2);
  const size_t o_logits = take((size_t)B * d.vocab * 4);
  const size_t o_best = take((size_t)B * 8);
  const size_t o_tok = take((size_t)B * 4);
  const size_t umma_rows = B >= kMmaMinBatch ? (size_t)B : 0;  // any batch that may take the tcgen05 path
  const size_t o_uacc = take(umma_rows * (d.n_in > d.d_model ? d.n_in : d.d_model) * 4);
  const size_t o_ucnt = take(umma_rows ? (size_t)kUmmaMaxTiles * 4 : 0);
  const int seen_words = (d.vocab + 31) / 32;
  const size_t o_seen = take((size_t)B * seen_words * 4);
  const size_t o_ctr = take((size_t)B * 8);
  const size_t o_layers = take(sizeof(LayerW) * d.n_layer);
  if (cudaMalloc(&e->work, off) != cudaSuccess)
    return cleanup(dfssm_fail(DFSSM_ERR_OOM, "cudaMalloc(%zu) for state/activations failed", off));
  e->work_bytes = off;
  char* W = e->work;
  e->ssm = reinterpret_cast<float*>(W + o_ssm);
  e->conv = reinterpret_cast<float*>(W + o_conv);
  e->x = reinterpret_cast<__half*>(W + o_x);
  e->xn = reinterpret_cast<__half*>(W + o_xn);
  e->q = reinterpret_cast<int8_t*>(W + o_q);
  e->xs = reinterpret_cast<__half*>(W + o_xs);
  e->qsum = reinterpret_cast<int*>(W + o_qsum);
  e->t = reinterpret_cast<__half*>(W + o_t);
  e->proj = reinterpret_cast<__half*>(W + o_proj);
  e->gated = reinterpret_cast<__half*>(W + o_gated);
  e->logits = reinterpret_cast<float*>(W + o_logits);
  e->best = reinterpret_cast<unsigned long long*>(W + o_best);
  e->tokens = reinterpret_cast<int*>(W + o_tok);
  e->sync = reinterpret_cast<unsigned int*>(W + o_sync);
  e->xch = reinterpret_cast<unsigned long long*>(W + o_xch);
  e->seen = reinterpret_cast<uint32_t*>(W + o_seen);
  e->uacc = umma_rows ? reinterpret_cast<int*>(W + o_uacc) : nullptr;
  e->ucnt = umma_rows ? reinterpret_cast<unsigned*>(W + o_ucnt) : nullptr;
  e->seen_words = seen_words;
  e->counters = reinterpret_cast<unsigned long long*>(W + o_ctr);
  e->d_layers = reinterpret_cast<LayerW*>(W + o_layers);
  ce = cudaMemset(e->work, 0, off);
  if (ce != cudaSuccess) return cleanup(dfssm_fail(DFSSM_ERR_CUDA, "state clear: %s", cudaGetErrorString(ce)));
  ce = cudaMemcpy(e->d_layers, e->layers.data(), sizeof(LayerW) * d.n_layer, cudaMemcpyHostToDevice);
  if (ce != cudaSuccess) return cleanup(dfssm_fail(DFSSM_ERR_CUDA, "layer table upload: %s", cudaGetErrorString(ce)));
  for (int g = 1; g < kMaxGroups; ++g)
    if (cudaStreamCreateWithFlags(&e->gs[g], cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->ev_join[g], cudaEventDisableTiming) != cudaSuccess)
      return cleanup(dfssm_fail(DFSSM_ERR_CUDA, "group stream creation failed"));
  if (cudaEventCreateWithFlags(&e->ev_fork, cudaEventDisableTiming) != cudaSuccess)
    return cleanup(dfssm_fail(DFSSM_ERR_CUDA, "event creation failed"));
  if (cudaStreamCreateWithFlags(&e->s, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&e->ev_in, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&e->ev_out, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&e->ev_cat, cudaEventDisableTiming) != cudaSuccess)
    return cleanup(dfssm_fail(DFSSM_ERR_CUDA, "stream/event creation failed"));
  // kernels that need more than 48 KB of dynamic shared memory
  const int gemv_smem = kGemvBT * kmax;
  const int head_smem = kHeadBT * d.d_model * 4;
  if (cudaFuncSetAttribute(proj_gemv_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemv_smem) != cudaSuccess ||
      cudaFuncSetAttribute(proj_gemv_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemv_smem) != cudaSuccess ||
      cudaFuncSetAttribute(lm_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, head_smem) != cudaSuccess)
    return cleanup(dfssm_fail(DFSSM_ERR_CUDA, "cudaFuncSetAttribute failed: %s", cudaGetErrorString(cudaGetLastError())));
  rc = persistent_init(e);
  if (rc) return cleanup(rc);
  *out = e;
  return DFSSM_OK;
}

}  // namespace

// ====================================================================== C ABI

extern "C" {

const char* dfssm_version(void) { return "dfssm-b200 0.1 (sm_100a)"; }

int dfssm_kernel_binary_version(int device, int* version) {
  if (!version) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  CU(cudaSetDevice(device));
  cudaFuncAttributes a;
  CU(cudaFuncGetAttributes(&a, reinterpret_cast<const void*>(embed_kernel)));
  *version = a.binaryVersion;
  return DFSSM_OK;
}
const char* dfssm_last_error(void) { return g_err.c_str(); }

int dfssm_create_from_memory(const void* image, size_t image_bytes, int device, int max_batch, dfssm_engine** out) {
  return build_engine(static_cast<const unsigned char*>(image), image_bytes, device, max_batch, out);
}

int dfssm_create_from_file(const char* path, int device, int max_batch, dfssm_engine** out) {
  if (!path) return dfssm_fail(DFSSM_ERR_ARG, "path is NULL");
  FILE* f = fopen(path, "rb");
  if (!f) return dfssm_fail(DFSSM_ERR_ARG, "cannot open %s", path);
  std::vector<unsigned char> buf;
  fseek(f, 0, SEEK_END);
  long n = ftell(f);
  fseek(f, 0, SEEK_SET);
  if (n < 0) {
    fclose(f);
    return dfssm_fail(DFSSM_ERR_ARG, "cannot size %s", path);
  }
  buf.resize((size_t)n);
  size_t got = n ? fread(buf.data(), 1, (size_t)n, f) : 0;
  fclose(f);
  if (got != (size_t)n) return dfssm_fail(DFSSM_ERR_FORMAT, "short read of %s", path);
  return build_engine(buf.data(), buf.size(), device, max_batch, out);
}

void dfssm_destroy(dfssm_engine* e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->gexec) cudaGraphExecDestroy(e->gexec);
  if (e->s) cudaStreamSynchronize(e->s);
  if (e->ev_in) cudaEventDestroy(e->ev_in);
  if (e->ev_out) cudaEventDestroy(e->ev_out);
  if (e->ev_cat) cudaEventDestroy(e->ev_cat);
  if (e->s) cudaStreamDestroy(e->s);
  for (int g = 1; g < kMaxGroups; ++g) {
    if (e->gs[g]) cudaStreamDestroy(e->gs[g]);
    if (e->ev_join[g]) cudaEventDestroy(e->ev_join[g]);
  }
  if (e->ev_fork) cudaEventDestroy(e->ev_fork);
  persistent_destroy(e);
  if (e->arena) cudaFree(e->arena);
  if (e->work) cudaFree(e->work);
  if (e->pf) cudaFree(e->pf);
  delete e;
}

int dfssm_get_dims(const dfssm_engine* e, dfssm_dims* out) {
  if (!e || !out) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  *out = e->d;
  return DFSSM_OK;
}

int dfssm_set_batch(dfssm_engine* e, int batch) {
  if (!e) return dfssm_fail(DFSSM_ERR_ARG, "NULL engine");
  if (batch < 1 || batch > e->max_batch)
    return dfssm_fail(DFSSM_ERR_ARG, "batch=%d outside [1, max_batch=%d]", batch, e->max_batch);
  e->batch = batch;
  return DFSSM_OK;
}

int dfssm_set_mode(dfssm_engine* e, int mode) {
  if (!e) return dfssm_fail(DFSSM_ERR_ARG, "NULL engine");
  if (mode < 0 || mode > 3) return dfssm_fail(DFSSM_ERR_ARG, "mode=%d unknown", mode);
  if (mode == 3 && !persistent_supported(e))
    return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "persistent step kernel not available for these dims/batch");
  e->mode = mode;
  return DFSSM_OK;
}

int dfssm_get_mode(const dfssm_engine* e, int* mode) {
  if (!e || !mode) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  *mode = effective_mode(e);
  return DFSSM_OK;
}

int dfssm_reset(dfssm_engine* e, void* stream) {
  if (!e) return dfssm_fail(DFSSM_ERR_ARG, "NULL engine");
  CU(cudaSetDevice(e->device));
  cudaStream_t us = static_cast<cudaStream_t>(stream);
  CU(cudaMemsetAsync(e->ssm, 0, e->ssm_layer * e->d.n_layer * 4, us));
  CU(cudaMemsetAsync(e->conv, 0, e->conv_layer * e->d.n_layer * 4, us));
  CU(cudaMemsetAsync(e->best, 0, (size_t)e->max_batch * 8, us));
  CU(cudaMemsetAsync(e->sync, 0, 32, us));
  CU(cudaMemsetAsync(e->seen, 0, (size_t)e->max_batch * e->seen_words * 4, us));
  CU(cudaMemsetAsync(e->counters, 0, (size_t)e->max_batch * 8, us));
  return DFSSM_OK;
}

int dfssm_reset_slots(dfssm_engine* e, int first, int count, void* stream) {
  if (!e) return dfssm_fail(DFSSM_ERR_ARG, "NULL engine");
  if (first < 0 || count < 1 || first + count > e->max_batch)
    return dfssm_fail(DFSSM_ERR_ARG, "slots [%d, %d) outside [0, max_batch=%d)", first, first + count, e->max_batch);
  CU(cudaSetDevice(e->device));
  cudaStream_t us = static_cast<cudaStream_t>(stream);
  const size_t hseq = e->ssm_layer / e->max_batch, cseq = e->conv_layer / e->max_batch;  // floats per sequence
  for (int l = 0; l < e->d.n_layer; ++l) {
    CU(cudaMemsetAsync(e->ssm + (size_t)l * e->ssm_layer + (size_t)first * hseq, 0, (size_t)count * hseq * 4, us));
    CU(cudaMemsetAsync(e->conv + (size_t)l * e->conv_layer + (size_t)first * cseq, 0, (size_t)count * cseq * 4, us));
  }
  CU(cudaMemsetAsync(e->seen + (size_t)first * e->seen_words, 0, (size_t)count * e->seen_words * 4, us));
  CU(cudaMemsetAsync(e->counters + first, 0, (size_t)count * 8, us));
  return DFSSM_OK;
}

int dfssm_step(dfssm_engine* e, const int32_t* tokens_dev, float* logits_dev, int32_t* next_tokens_dev,
               void* stream) {
  if (!e) return dfssm_fail(DFSSM_ERR_ARG, "NULL engine");
  CU(cudaSetDevice(e->device));
  cudaStream_t us = static_cast<cudaStream_t>(stream);
  const int mode = effective_mode(e);
  if (mode == 3 && !persistent_supported(e))
    return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "persistent step kernel not available for batch %d", e->batch);
  const bool sampling = e->s_temp > 0.f;
  if (mode == 3 && e->order_valid && e->order_s == us) {
    // all earlier engine work is already ordered into this stream: run the step on it directly,
    // without the two cross-stream event hops (a host round trip of the step path saves ~5%)
    if (tokens_dev) CU(cudaMemcpyAsync(e->tokens, tokens_dev, (size_t)e->batch * 4, cudaMemcpyDeviceToDevice, us));
    if (sampling) {
      mark_seen_kernel<<<(e->batch + 127) / 128, 128, 0, us>>>(e->tokens, e->batch, e->d.vocab, e->seen, e->seen_words);
      CHECK_LAUNCH();
    }
    int rc;
    if ((rc = launch_persistent_step(e, us))) return rc;
    if (sampling &&
        (rc = dfssm_sample(e->logits, e->batch, e->d.vocab, e->seen, e->s_temp, e->s_top_p, e->s_rep, e->s_seed,
                           reinterpret_cast<uint64_t*>(e->counters), e->tokens, nullptr, nullptr, us)))
      return rc;
    if (logits_dev)
      CU(cudaMemcpyAsync(logits_dev, e->logits, (size_t)e->batch * e->d.vocab * 4, cudaMemcpyDeviceToDevice, us));
    if (next_tokens_dev)
      CU(cudaMemcpyAsync(next_tokens_dev, e->tokens, (size_t)e->batch * 4, cudaMemcpyDeviceToDevice, us));
    return DFSSM_OK;
  }
  CU(engine_stream_after(e, us));
  if (tokens_dev)
    CU(cudaMemcpyAsync(e->tokens, tokens_dev, (size_t)e->batch * 4, cudaMemcpyDeviceToDevice, e->s));
  if (sampling) {  // the input tokens join each sequence's seen set before the penalty applies
    mark_seen_kernel<<<(e->batch + 127) / 128, 128, 0, e->s>>>(e->tokens, e->batch, e->d.vocab, e->seen, e->seen_words);
    CHECK_LAUNCH();
  }
  int rc;
  if (mode == 2) {
    if ((rc = enqueue_step(e, 1, e->s))) return rc;
  } else if (mode == 3) {
    if ((rc = launch_persistent_step(e, e->s))) return rc;
  } else {
    if ((rc = ensure_graph(e, mode))) return rc;
    CU(cudaGraphLaunch(e->gexec, e->s));
  }
  if (sampling &&
      (rc = dfssm_sample(e->logits, e->batch, e->d.vocab, e->seen, e->s_temp, e->s_top_p, e->s_rep, e->s_seed,
                         reinterpret_cast<uint64_t*>(e->counters), e->tokens, nullptr, nullptr, e->s)))
    return rc;
  if (logits_dev)
    CU(cudaMemcpyAsync(logits_dev, e->logits, (size_t)e->batch * e->d.vocab * 4, cudaMemcpyDeviceToDevice, e->s));
  if (next_tokens_dev)
    CU(cudaMemcpyAsync(next_tokens_dev, e->tokens, (size_t)e->batch * 4, cudaMemcpyDeviceToDevice, e->s));
  CU(cudaEventRecord(e->ev_out, e->s));
  CU(cudaStreamWaitEvent(us, e->ev_out, 0));
  e->order_s = us;
  e->order_valid = true;
  return DFSSM_OK;
}

int dfssm_step_host(dfssm_engine* e, const int32_t* tokens_host, float* logits_host, int32_t* next_tokens_host,
                    void* stream) {
  if (!e) return dfssm_fail(DFSSM_ERR_ARG, "NULL engine");
  CU(cudaSetDevice(e->device));
  cudaStream_t us = static_cast<cudaStream_t>(stream);
  if (tokens_host) CU(cudaMemcpyAsync(e->tokens, tokens_host, (size_t)e->batch * 4, cudaMemcpyHostToDevice, us));
  int rc = dfssm_step(e, nullptr, nullptr, nullptr, stream);
  if (rc) return rc;
  if (logits_host)
    CU(cudaMemcpyAsync(logits_host, e->logits, (size_t)e->batch * e->d.vocab * 4, cudaMemcpyDeviceToHost, us));
  if (next_tokens_host)
    CU(cudaMemcpyAsync(next_tokens_host, e->tokens, (size_t)e->batch * 4, cudaMemcpyDeviceToHost, us));
  CU(cudaStreamSynchronize(us));
  return DFSSM_OK;
}

int dfssm_check_finite(dfssm_engine* e, void* stream) {
  if (!e) return dfssm_fail(DFSSM_ERR_ARG, "NULL engine");
  CU(cudaSetDevice(e->device));
  std::vector<float> h((size_t)e->batch * e->d.vocab);
  CU(cudaMemcpyAsync(h.data(), e->logits, h.size() * 4, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)));
  CU(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  unsigned sync_err = 0, umma_err = 0;
  CU(cudaMemcpy(&sync_err, e->sync + 3, 4, cudaMemcpyDeviceToHost));
  CU(cudaMemcpyFromSymbol(&umma_err, g_umma_err, 4));
  if (umma_err)
    return dfssm_fail(DFSSM_ERR_STATE, "a per-op projection or LM-head kernel recorded a timed-out wait (code %u)",
                      umma_err);
  if (sync_err)
    return dfssm_fail(DFSSM_ERR_STATE, "persistent step kernel recorded a timed-out wait (code %u)", sync_err);
  for (size_t i = 0; i < h.size(); ++i)
    if (!std::isfinite(h[i])) return dfssm_fail(DFSSM_ERR_NUMERIC, "non-finite logit at flat index %zu", i);
  return DFSSM_OK;
}

int dfssm_state_ptrs(dfssm_engine* e, int layer, float** ssm, float** conv) {
  if (!e || !ssm || !conv) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  if (layer < 0 || layer >= e->d.n_layer) return dfssm_fail(DFSSM_ERR_ARG, "layer %d out of range", layer);
  *ssm = e->ssm + (size_t)layer * e->ssm_layer;
  *conv = e->conv + (size_t)layer * e->conv_layer;
  return DFSSM_OK;
}

int dfssm_get_buffer(dfssm_engine* e, const char* name, void** ptr, size_t* bytes) {
  if (!e || !name || !ptr || !bytes) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  const dfssm_dims& d = e->d;
  const size_t B = e->max_batch;
  if (!strcmp(name, "x")) { *ptr = e->x; *bytes = B * d.d_model * 2; }
  else if (!strcmp(name, "proj")) { *ptr = e->proj; *bytes = B * d.n_in * 2; }
  else if (!strcmp(name, "gated")) { *ptr = e->gated; *bytes = B * d.d_inner * 2; }
  else if (!strcmp(name, "logits")) { *ptr = e->logits; *bytes = B * d.vocab * 4; }
  else if (!strcmp(name, "tokens")) { *ptr = e->tokens; *bytes = B * 4; }
  else if (!strcmp(name, "q")) { *ptr = e->q; *bytes = B * (d.d_model > d.d_inner ? d.d_model : d.d_inner); }
  else if (!strcmp(name, "xs")) { *ptr = e->xs; *bytes = B * 2; }
  else return dfssm_fail(DFSSM_ERR_ARG, "unknown buffer '%s'", name);
  return DFSSM_OK;
}

int dfssm_weight_ptr(dfssm_engine* e, int layer, const char* name, void** ptr, size_t* bytes) {
  if (!e || !name || !ptr || !bytes) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  const dfssm_dims& d = e->d;
  if (layer < 0) {
    if (!strcmp(name, "emb_q")) { *ptr = const_cast<int8_t*>(e->Eq); *bytes = (size_t)d.vocab * d.d_model; }
    else if (!strcmp(name, "emb_s")) { *ptr = const_cast<float*>(e->Es); *bytes = (size_t)d.vocab * 4; }
    else if (!strcmp(name, "norm_f")) { *ptr = const_cast<float*>(e->norm_f); *bytes = (size_t)d.d_model * 4; }
    else return dfssm_fail(DFSSM_ERR_ARG, "unknown model weight '%s'", name);
    return DFSSM_OK;
  }
  if (layer >= d.n_layer) return dfssm_fail(DFSSM_ERR_ARG, "layer %d out of range", layer);
  const LayerW& L = e->layers[layer];
  auto proj = [&](const ProjW& p, const char* f) -> int {
    if (!strcmp(f, "bits")) { *ptr = const_cast<uint32_t*>(p.bits); *bytes = (size_t)p.N * (p.K / 32) * 4; }
    else if (!strcmp(f, "scale")) { *ptr = const_cast<__half*>(p.scale); *bytes = (size_t)p.N * 2; }
    else if (!strcmp(f, "lora_A")) { *ptr = const_cast<__half*>(p.A16); *bytes = (size_t)p.N * kRank * 2; }
    else if (!strcmp(f, "lora_B")) { *ptr = const_cast<__half*>(p.B16); *bytes = (size_t)kRank * p.K * 2; }
    else return 0;
    return 1;
  };
  if (!strncmp(name, "in_", 3) && proj(L.in, name + 3)) return DFSSM_OK;
  if (!strncmp(name, "out_", 4) && proj(L.out, name + 4)) return DFSSM_OK;
  if (!strcmp(name, "conv_w")) { *ptr = const_cast<__half*>(L.conv_w); *bytes = (size_t)d.d_xbc * 4 * 2; }
  else if (!strcmp(name, "conv_b")) { *ptr = const_cast<__half*>(L.conv_b); *bytes = (size_t)d.d_xbc * 2; }
  else if (!strcmp(name, "A_log")) { *ptr = const_cast<float*>(L.A_log); *bytes = (size_t)d.nheads * 4; }
  else if (!strcmp(name, "D")) { *ptr = const_cast<float*>(L.Dp); *bytes = (size_t)d.nheads * 4; }
  else if (!strcmp(name, "dt_bias")) { *ptr = const_cast<float*>(L.dt_bias); *bytes = (size_t)d.nheads * 4; }
  else if (!strcmp(name, "norm_w")) { *ptr = const_cast<float*>(L.norm_w); *bytes = (size_t)d.d_inner * 4; }
  else if (!strcmp(name, "ln_w")) { *ptr = const_cast<float*>(L.ln_w); *bytes = (size_t)d.d_model * 4; }
  else return dfssm_fail(DFSSM_ERR_ARG, "unknown layer weight '%s'", name);
  return DFSSM_OK;
}

int dfssm_layer_step(dfssm_engine* e, int layer, void* stream) {
  if (!e) return dfssm_fail(DFSSM_ERR_ARG, "NULL engine");
  if (layer < 0 || layer >= e->d.n_layer) return dfssm_fail(DFSSM_ERR_ARG, "layer %d out of range", layer);
  CU(cudaSetDevice(e->device));
  if (effective_mode(e) == 3)
    return launch_persistent_layers(e, layer, layer + 1, 1, 0, static_cast<cudaStream_t>(stream));
  return enqueue_layer(e, layer, static_cast<cudaStream_t>(stream), Group{0, e->batch});
}

int dfssm_debug_set_wait_limit(dfssm_engine* e, unsigned polls) {
  if (!e) return dfssm_fail(DFSSM_ERR_ARG, "NULL engine");
  return persistent_debug_wait_limit(e, polls);
}

int dfssm_debug_skew_next_step(dfssm_engine* e) {
  if (!e) return dfssm_fail(DFSSM_ERR_ARG, "NULL engine");
  return persistent_debug_skew(e);
}

size_t dfssm_trace_entries(const dfssm_engine* e) { return e ? persistent_trace_entries(e) : 0; }

int dfssm_trace_step(dfssm_engine* e, unsigned long long* trace_dev, void* stream) {
  if (!e || !trace_dev) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  CU(cudaSetDevice(e->device));
  return launch_persistent_traced(e, trace_dev, static_cast<cudaStream_t>(stream));
}

size_t dfssm_scaffold_gemm_workspace(int M, int K) {
  if (M <= 0 || K <= 0) return 0;
  return align256((size_t)M * K) + align256((size_t)M * 4) + align256((size_t)M * 2) + align256((size_t)M * kRank * 2);
}

int dfssm_scaffold_gemm(const uint32_t* packed, const int8_t* q, int M, int N, int K, int32_t* acc, void* workspace,
                        void* stream) {
  if (!packed || !q || !acc || !workspace) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  if (M < 1 || N < 1 || K < 128 || K % 128 || K > 65536) return dfssm_fail(DFSSM_ERR_ARG, "bad sizes M=%d N=%d K=%d", M, N, K);
  if (((uintptr_t)packed | (uintptr_t)workspace) & 15) return dfssm_fail(DFSSM_ERR_ARG, "packed/workspace must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProjW p{};
  p.bits = packed;
  p.N = N;
  p.K = K;
  const int rows_per_cta = 2 * (kGemvThreads / 32);
  // mma.sync from one row (measured at the 1.3B in_proj shape: M = 1 in ~6.8 us against 9.8 us on the
  // GEMV, whose activation staging and weight loads form one more latency chain); DFSSM_GEMM_MMA_MIN
  // overrides
  static const int mma_from = [] {
    const char* v = getenv("DFSSM_GEMM_MMA_MIN");
    return v ? atoi(v) : 1;
  }();
  if (M < mma_from || !mma_rg(N, K)) {  // the GEMV permutes and sums the rows itself: one launch
    if ((uintptr_t)q & 15) return dfssm_fail(DFSSM_ERR_ARG, "q must be 16-byte aligned");
    const size_t sm = (size_t)kGemvBT * K;
    if (sm > 48 * 1024) CU(ensure_smem(reinterpret_cast<const void*>(proj_gemv_kernel<4>), sm));
    proj_gemv_kernel<4><<<(N + rows_per_cta - 1) / rows_per_cta, kGemvThreads, sm, s>>>(
        p, q, nullptr, nullptr, nullptr, M, reinterpret_cast<__half*>(acc), N, nullptr, nullptr, nullptr, 0, 0);
    CHECK_LAUNCH();
    return DFSSM_OK;
  }
  char* ws = static_cast<char*>(workspace);
  int8_t* qp = reinterpret_cast<int8_t*>(ws);
  int* qsum = reinterpret_cast<int*>(ws + align256((size_t)M * K));
  permute_q_kernel<<<M, kPrepThreads, 0, s>>>(q, K, qp, qsum);
  CHECK_LAUNCH();
  return launch_mma<2>(p, M, qp, qsum, nullptr, nullptr, acc, N, nullptr, nullptr, nullptr, 0, 0, s);
}

int dfssm_conv_step(float* conv_state, void* xbc_f16, int ld_xbc, const void* conv_w_f16, const void* conv_b_f16,
                    int batch, int d_xbc, void* stream) {
  if (!conv_state || !xbc_f16 || !conv_w_f16 || !conv_b_f16) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  if (batch < 1 || d_xbc < 1 || ld_xbc < d_xbc) return dfssm_fail(DFSSM_ERR_ARG, "bad sizes");
  conv_step_kernel<<<dim3((d_xbc + 255) / 256, batch), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      conv_state, static_cast<__half*>(xbc_f16), ld_xbc, static_cast<const __half*>(conv_w_f16),
      static_cast<const __half*>(conv_b_f16), d_xbc);
  CHECK_LAUNCH();
  return DFSSM_OK;
}

int dfssm_ssm_step(const void* xbc_f16, int ld_xbc, const void* dt_f16, int ld_dt, const float* dt_bias,
                   const float* A_log, const float* D, float* h_state, void* y_f16, int ld_y, int batch, int nheads,
                   int headdim, int d_state, void* stream) {
  if (!xbc_f16 || !dt_f16 || !dt_bias || !A_log || !D || !h_state || !y_f16) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  if (headdim != DFSSM_HEADDIM || d_state != DFSSM_DSTATE)
    return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "headdim=%d d_state=%d (built for 64/128)", headdim, d_state);
  if (batch < 1 || nheads < 1) return dfssm_fail(DFSSM_ERR_ARG, "bad sizes");
  if ((uintptr_t)h_state & 15) return dfssm_fail(DFSSM_ERR_ARG, "h_state must be 16-byte aligned");
  if (ld_xbc % 4 || ((uintptr_t)xbc_f16 & 7))
    return dfssm_fail(DFSSM_ERR_ARG, "xbc rows must start on 8-byte boundaries (ld_xbc %% 4 == 0)");
  const int d_inner = nheads * headdim;
  ssm_gate_kernel<<<dim3(nheads, batch), kSsmThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(xbc_f16), ld_xbc, static_cast<const __half*>(dt_f16), ld_dt, nullptr, 0, d_inner,
      d_state, nheads, dt_bias, A_log, D, h_state, static_cast<__half*>(y_f16), ld_y);
  CHECK_LAUNCH();
  return DFSSM_OK;
}

int dfssm_rmsnorm_quantize(const void* x_f16, const float* norm_w, int batch, int K, void* xn_f16, void* scale_f16,
                           int8_t* q, void* stream) {
  if (!x_f16 || !norm_w || !xn_f16 || !scale_f16 || !q) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  if (batch < 1) return dfssm_fail(DFSSM_ERR_ARG, "batch %d < 1", batch);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __half* x = static_cast<const __half*>(x_f16);
  __half* xn = static_cast<__half*>(xn_f16);
  __half* xs = static_cast<__half*>(scale_f16);
#define DFSSM_RQ(n)                                                                                   \
  if (K == 512 * n) {                                                                                 \
    rmsnorm_quant_kernel<n><<<batch, kPrepFastThreads, 0, s>>>(x, K, norm_w, xn, xs, q);              \
    CHECK_LAUNCH();                                                                                   \
    return DFSSM_OK;                                                                                  \
  }
  DFSSM_RQ(1)
  DFSSM_RQ(2)
  DFSSM_RQ(4)
  DFSSM_RQ(5)
  DFSSM_RQ(8)
  DFSSM_RQ(10)
#undef DFSSM_RQ
  return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "K=%d (built for 512 x {1, 2, 4, 5, 8, 10})", K);
}

size_t dfssm_lm_head_workspace(int batch) { return batch > 0 ? align256((size_t)batch * 8) : 0; }

int dfssm_lm_head_argmax(const int8_t* E_q, const float* E_s, int vocab, int d, const void* x_f16, int batch,
                         float* logits, int32_t* next, void* workspace, void* stream) {
  if (!E_q || !E_s || !x_f16 || !next || !workspace) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  if (vocab < 1 || batch < 1 || d < 16 || d % 16) return dfssm_fail(DFSSM_ERR_ARG, "bad sizes");
  if ((uintptr_t)E_q & 15 || (d % 16)) return dfssm_fail(DFSSM_ERR_ARG, "E_q rows must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned long long* best = static_cast<unsigned long long*>(workspace);
  CU(cudaMemsetAsync(best, 0, (size_t)batch * 8, s));
  float* lg = logits;
  if (!lg) return dfssm_fail(DFSSM_ERR_ARG, "logits output is required by this build");
  const size_t sm = (size_t)kHeadBT * d * sizeof(float);
  if (sm > 48 * 1024) CU(ensure_smem(reinterpret_cast<const void*>(lm_head_kernel), sm));
  int sms = 148;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (batch >= kMmaMinBatch && d % (64 * kHeadMmaU) == 0) {
    int rc2 = launch_head_mma(E_q, E_s, vocab, d, static_cast<const __half*>(x_f16), batch, lg, best, sms, s);
    if (rc2) return rc2;
  } else {
    lm_head_kernel<<<sms * 4, kHeadThreads, sm, s>>>(E_q, E_s, vocab, d, static_cast<const __half*>(x_f16), batch, lg,
                                                      best);
  }
  CHECK_LAUNCH();
  finalize_kernel<<<(batch + 127) / 128, 128, 0, s>>>(best, batch, reinterpret_cast<int*>(next));
  CHECK_LAUNCH();
  return DFSSM_OK;
}

}  // extern "C"

// ====================================================================== allocation-free scaffold GEMM
//
// Some callers of this library cannot allocate device memory at the point where they need a
// scaffold GEMM: code running inside a host-side allocator callback, plug-in hosts whose
// memory pool forbids foreign cudaMalloc calls, or real-time loops where an allocation could
// block or fail.  dfssm_scaffold_gemm_noalloc serves them: the scratch it needs (the
// activations in the GEMV's permuted byte order plus their row sums) lives in a fixed
// file-scope device array instead of caller- or library-allocated memory.
namespace {

constexpr size_t kNoAllocMaxQBytes = size_t(2) << 20;  // M * K <= 2 MiB of int8 activations
constexpr int kNoAllocMaxRows = 2048;                   // M <= 2048
constexpr size_t kNoAllocQsumOff = kNoAllocMaxQBytes;   // 256-aligned
constexpr size_t kNoAllocBytes = kNoAllocMaxQBytes + kNoAllocMaxRows * sizeof(int);

// Every GPU that loads this library holds this array (2 MiB + 8 KiB) until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device.  In host code the array's name is
// only a host-side stand-in, so the real address is looked up once per device (with that device
// current) and cached.
int noalloc_scratch(void** out) {
  int dev = 0;
  CU(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices) return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    CU(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return DFSSM_OK;
}

}  // namespace

extern "C" int dfssm_scaffold_gemm_noalloc(const uint32_t* packed, const int8_t* q, int M, int N, int K,
                                           int32_t* acc, void* stream) {
  if (!packed || !q || !acc) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  if (M < 1 || N < 1 || K < 128 || K % 128 || K > 65536) return dfssm_fail(DFSSM_ERR_ARG, "bad sizes M=%d N=%d K=%d", M, N, K);
  if (M > kNoAllocMaxRows || (size_t)M * (size_t)K > kNoAllocMaxQBytes)
    return dfssm_fail(DFSSM_ERR_ARG,
                      "M=%d K=%d exceeds the fixed scratch of dfssm_scaffold_gemm_noalloc (M*K <= %zu, M <= %d); "
                      "use dfssm_scaffold_gemm with a caller workspace",
                      M, K, kNoAllocMaxQBytes, kNoAllocMaxRows);
  if ((uintptr_t)packed & 15) return dfssm_fail(DFSSM_ERR_ARG, "packed must be 16-byte aligned");
  void* ws = nullptr;
  int rc = noalloc_scratch(&ws);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int8_t* qp = static_cast<int8_t*>(ws);
  int* qsum = reinterpret_cast<int*>(static_cast<char*>(ws) + kNoAllocQsumOff);
  // Both scratch regions are fully rewritten before they are read, so nothing needs clearing.
  permute_q_kernel<<<M, kPrepThreads, 0, s>>>(q, K, qp, qsum);
  CHECK_LAUNCH();
  ProjW p{};
  p.bits = packed;
  p.N = N;
  p.K = K;
  // the same kernel choice as dfssm_scaffold_gemm: the tensor-core kernels need no scratch beyond
  // the permuted activations and their sums (a split-K tcgen05 launch zeroes `acc` and adds into it)
  if (M >= kMmaMinBatch && mma_rg(N, K))
    return launch_mma<2>(p, M, qp, qsum, nullptr, nullptr, acc, N, nullptr, nullptr, nullptr, 0, 0, s);
  const size_t sm = (size_t)kGemvBT * K;
  if (sm > 48 * 1024) CU(ensure_smem(reinterpret_cast<const void*>(proj_gemv_kernel<2>), sm));
  const int rows_per_cta = 2 * (kGemvThreads / 32);
  proj_gemv_kernel<2><<<(N + rows_per_cta - 1) / rows_per_cta, kGemvThreads, sm, s>>>(
      p, qp, qsum, nullptr, nullptr, M, reinterpret_cast<__half*>(acc), N, nullptr, nullptr, nullptr, 0, 0);
  CHECK_LAUNCH();
  return DFSSM_OK;
}

// ------------------------------------------------------------------ division self-test

namespace {
__global__ void selftest_division_kernel(unsigned long long* mismatch) {
  const unsigned short sb = (unsigned short)(blockIdx.x + 1);  // divisor: every positive finite fp16
  const float b = __half2float(__ushort_as_half(sb));
  const float rb = __frcp_rn(b);
  unsigned long long m32 = 0, m16 = 0;
  for (unsigned a16 = threadIdx.x; a16 < 0x10000u; a16 += blockDim.x) {
    if ((a16 & 0x7C00u) == 0x7C00u) continue;  // inf / NaN
    const float a = __half2float(__ushort_as_half((unsigned short)a16));
    const float q = div_rn_rcp(a, b, rb);
    const float ref = __fdiv_rn(a, b);
    // zeros compare equal whatever their sign: -0 / b gives +0 here, and both quantise to 0
    m32 += q != ref || (q != 0.f && __float_as_uint(q) != __float_as_uint(ref));
    m16 += __half_as_ushort(__float2half_rn(q)) != __half_as_ushort(__float2half_rn(ref)) && q != 0.f;
  }
  if (m32) atomicAdd(mismatch, m32);
  if (m16) atomicAdd(mismatch + 1, m16);
}
}  // namespace

int dfssm_selftest_division(int device, unsigned long long* mismatch) {
  if (!mismatch) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  CU(cudaSetDevice(device));
  unsigned long long* d = nullptr;
  CU(cudaMalloc(&d, 16));
  cudaError_t ce = cudaMemset(d, 0, 16);
  if (ce == cudaSuccess) {
    selftest_division_kernel<<<0x7BFF, 256>>>(d);
    ce = cudaGetLastError();
  }
  if (ce == cudaSuccess) ce = cudaMemcpy(mismatch, d, 16, cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (ce != cudaSuccess) return dfssm_fail(DFSSM_ERR_CUDA, "division self-test: %s", cudaGetErrorString(ce));
  return DFSSM_OK;
}

// ------------------------------------------------------------------ sampling epilogue

int dfssm_sample(const float* logits, int batch, int vocab, uint32_t* seen_bits, float temperature, float top_p,
                 float rep_penalty, uint64_t seed, uint64_t* counters, int32_t* next, float* kept_mass,
                 int32_t* kept_count, void* stream) {
  if (!logits || !seen_bits || !counters || !next) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  if (batch < 1 || vocab < 1) return dfssm_fail(DFSSM_ERR_ARG, "batch %d vocab %d", batch, vocab);
  if (!(temperature > 0.f) || !(rep_penalty > 0.f) || !(top_p >= 0.f))
    return dfssm_fail(DFSSM_ERR_ARG, "temperature and rep_penalty must be > 0, top_p >= 0");
  const size_t sm = (size_t)vocab * 4;
  int dev = 0, max_sm = 0;
  CU(cudaGetDevice(&dev));
  CU(cudaDeviceGetAttribute(&max_sm, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  if (sm + 1024 > (size_t)max_sm)
    return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "vocab %d needs %zu bytes of shared memory (max %d)", vocab, sm, max_sm);
  CU(ensure_smem(reinterpret_cast<const void*>(sample_kernel), sm));
  sample_kernel<<<batch, kSampleThreads, sm, static_cast<cudaStream_t>(stream)>>>(
      logits, vocab, seen_bits, (vocab + 31) / 32, temperature, top_p, rep_penalty,
      (unsigned long long)seed, reinterpret_cast<unsigned long long*>(counters), next, kept_mass, kept_count);
  CHECK_LAUNCH();
  return DFSSM_OK;
}

int dfssm_set_sampling(dfssm_engine* e, float temperature, float top_p, float rep_penalty, uint64_t seed) {
  if (!e) return dfssm_fail(DFSSM_ERR_ARG, "NULL engine");
  if (temperature > 0.f && (!(rep_penalty > 0.f) || !(top_p >= 0.f)))
    return dfssm_fail(DFSSM_ERR_ARG, "rep_penalty must be > 0 and top_p >= 0");
  if (temperature > 0.f && (size_t)e->d.vocab * 4 + 1024 > 232448)
    return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "vocab %d too large for the sampling epilogue", e->d.vocab);
  e->s_temp = temperature > 0.f ? temperature : 0.f;
  e->s_top_p = top_p;
  e->s_rep = rep_penalty;
  e->s_seed = seed;
  return DFSSM_OK;
}

// ------------------------------------------------------------------ prompt prefill

namespace {

struct PrefillBufs {
  __half *x, *xn, *xs, *t, *proj, *gated;
  int8_t* q;
  int* qsum;
  int* tok;
  UmmaScratch us;
};

int prefill_bufs(dfssm_engine* e, int rows, PrefillBufs& P) {
  const dfssm_dims& d = e->d;
  const size_t kmax = d.d_inner > d.d_model ? d.d_inner : d.d_model;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  const size_t ox = take((size_t)rows * d.d_model * 2), oxn = take((size_t)rows * kmax * 2),
               oq = take((size_t)rows * kmax), oxs = take((size_t)rows * 2), oqs = take((size_t)rows * 4),
               ot = take((size_t)rows * kRank * 2), op = take((size_t)rows * d.n_in * 2),
               og = take((size_t)rows * d.d_inner * 2), otk = take((size_t)rows * 4),
               oua = take((size_t)rows * (d.n_in > d.d_model ? d.n_in : d.d_model) * 4),
               ouc = take((size_t)kUmmaMaxTiles * 4);
  if (off > e->pf_bytes) {
    if (e->pf) CU(cudaFree(e->pf));
    e->pf = nullptr;
    e->pf_bytes = 0;
    if (cudaMalloc(&e->pf, off) != cudaSuccess)
      return dfssm_fail(DFSSM_ERR_OOM, "cudaMalloc(%zu) for prefill rows failed", off);
    CU(cudaMemset(e->pf, 0, off));  // the split-K scratch starts (and stays) zero
    e->pf_bytes = off;
  }
  char* W = e->pf;
  P = PrefillBufs{reinterpret_cast<__half*>(W + ox), reinterpret_cast<__half*>(W + oxn), reinterpret_cast<__half*>(W + oxs),
                  reinterpret_cast<__half*>(W + ot), reinterpret_cast<__half*>(W + op), reinterpret_cast<__half*>(W + og),
                  reinterpret_cast<int8_t*>(W + oq), reinterpret_cast<int*>(W + oqs), reinterpret_cast<int*>(W + otk),
                  UmmaScratch{reinterpret_cast<int*>(W + oua), reinterpret_cast<unsigned*>(W + ouc)}};
  return DFSSM_OK;
}

// All layers over the B x T prompt rows of one chunk; the state carries over from the previous chunk.
int prefill_chunk(dfssm_engine* e, const PrefillBufs& P, int T, cudaStream_t s) {
  const dfssm_dims& d = e->d;
  const int B = e->batch, R = B * T;
  const RowBufs rb{P.xn, P.q, P.xs, P.qsum, P.t};
  embed_rows_kernel<<<R, 256, 0, s>>>(P.tok, e->Eq, e->Es, d.d_model, d.vocab, P.x);
  CHECK_LAUNCH();
  // two CTAs per (head, sequence) while one each would leave SMs idle (the B/C conv is repeated)
  const int split = d.nheads * B < e->sm_count ? 2 : 1;
  // the chunk's recurrence in the SSD matrix form on the tensor cores from 32 tokens (measured at the
  // 1.3B shape: 7% faster per prompt at 64 tokens, 3% slower at 16); DFSSM_PREFILL_SCAN=1 / 0 forces
  // the token-by-token loop / the SSD form
  static const int force = [] {
    const char* v = getenv("DFSSM_PREFILL_SCAN");
    return v ? atoi(v) : -1;
  }();
  const bool ssd = force == 1 ? false : (force == 0 ? true : T >= 32);
  const size_t sm = prefill_scan_smem(T, d.d_state, split, ssd);
  const void* scan = split == 2 ? (ssd ? reinterpret_cast<const void*>(prefill_scan_kernel<2, true>)
                                       : reinterpret_cast<const void*>(prefill_scan_kernel<2, false>))
                                : (ssd ? reinterpret_cast<const void*>(prefill_scan_kernel<1, true>)
                                       : reinterpret_cast<const void*>(prefill_scan_kernel<1, false>));
  CU(ensure_smem(scan, sm));
  int rc;
  for (int l = 0; l < d.n_layer; ++l) {
    const LayerW& L = e->layers[l];
    if ((rc = launch_prep(e, P.x, d.d_model, L.ln_w, 1, &L.in, s, Group{0, R}, rb))) return rc;
    if ((rc = launch_mma<3>(L.in, R, P.q, P.qsum, P.xs, P.t, P.proj, d.n_in, nullptr, nullptr, nullptr, d.d_inner,
                            d.d_xbc, s, P.us)))
      return rc;
    void* args[] = {const_cast<__half**>(&P.proj), const_cast<int*>(&d.n_in), &T, const_cast<int*>(&d.d_inner),
                    const_cast<int*>(&d.d_state), const_cast<int*>(&d.nheads), const_cast<__half**>(&L.conv_w),
                    const_cast<__half**>(&L.conv_b), const_cast<float**>(&L.dt_bias), const_cast<float**>(&L.A_log),
                    const_cast<float**>(&L.Dp), nullptr, nullptr, const_cast<__half**>(&P.gated)};
    float* cs_l = e->conv + (size_t)l * e->conv_layer;
    float* hs_l = e->ssm + (size_t)l * e->ssm_layer;
    args[11] = &cs_l;
    args[12] = &hs_l;
    CU(cudaLaunchKernel(scan, dim3(d.nheads * split, B), dim3(kScanThreads), args, sm, s));
    CHECK_LAUNCH();
    if ((rc = launch_prep(e, P.gated, d.d_inner, L.norm_w, 1, &L.out, s, Group{0, R}, rb))) return rc;
    if ((rc = launch_mma<1>(L.out, R, P.q, P.qsum, P.xs, P.t, P.x, d.d_model, nullptr, nullptr, nullptr, d.d_inner,
                            d.d_xbc, s, P.us)))
      return rc;
  }
  return DFSSM_OK;
}

}  // namespace

namespace {

// The prefill of dfssm_prefill for engine `e`, which may be a slot view of `owner` (the engine
// that owns the prompt-row buffers).
int prefill_impl(dfssm_engine* e, dfssm_engine* owner, const int32_t* tokens_dev, int T, float* logits_dev,
                 int32_t* next_tokens_dev, void* stream) {
  if (!e || !tokens_dev) return dfssm_fail(DFSSM_ERR_ARG, "NULL argument");
  if (T < 1) return dfssm_fail(DFSSM_ERR_ARG, "prompt length %d", T);
  CU(cudaSetDevice(e->device));
  cudaStream_t us = static_cast<cudaStream_t>(stream);
  const dfssm_dims& d = e->d;
  const int B = e->batch;
  const int Tc = T < kScanMaxT ? T : kScanMaxT;
  const bool batched = B * (T < Tc ? T : Tc) >= kMmaMinBatch && mma_rg(d.n_in, d.d_model) && mma_rg(d.d_model, d.d_inner) &&
                       prefill_scan_smem(Tc, d.d_state, 1, true) <= 227 * 1024;
  if (!batched) {  // too few rows for the batched kernels: token by token through dfssm_step
    for (int t = 0; t < T; ++t) {
      CU(cudaMemcpy2DAsync(e->tokens, 4, tokens_dev + t, (size_t)T * 4, 4, B, cudaMemcpyDeviceToDevice, us));
      int rc = dfssm_step(e, nullptr, t == T - 1 ? logits_dev : nullptr, t == T - 1 ? next_tokens_dev : nullptr, stream);
      if (rc) return rc;
    }
    return DFSSM_OK;
  }
  PrefillBufs P;
  int rc;
  if ((rc = prefill_bufs(owner, B * Tc, P))) return rc;
  CU(engine_stream_after(e, us));
  for (int t0 = 0; t0 < T; t0 += Tc) {
    const int tc = T - t0 < Tc ? T - t0 : Tc;
    if (B * tc < kMmaMinBatch) {  // a short tail chunk: token by token
      for (int t = t0; t < T; ++t) {
        CU(cudaMemcpy2DAsync(e->tokens, 4, tokens_dev + t, (size_t)T * 4, 4, B, cudaMemcpyDeviceToDevice, e->s));
        CU(cudaEventRecord(e->ev_out, e->s));
        CU(cudaStreamWaitEvent(us, e->ev_out, 0));
        if ((rc = dfssm_step(e, nullptr, t == T - 1 ? logits_dev : nullptr, t == T - 1 ? next_tokens_dev : nullptr,
                             stream)))
          return rc;
        CU(cudaEventRecord(e->ev_in, us));
        CU(cudaStreamWaitEvent(e->s, e->ev_in, 0));
      }
      CU(cudaEventRecord(e->ev_out, e->s));
      CU(cudaStreamWaitEvent(us, e->ev_out, 0));
      return DFSSM_OK;
    }
    CU(cudaMemcpy2DAsync(P.tok, (size_t)tc * 4, tokens_dev + t0, (size_t)T * 4, (size_t)tc * 4, B,
                         cudaMemcpyDeviceToDevice, e->s));
    if (e->s_temp > 0.f) {
      mark_seen_rows_kernel<<<(B * tc + 127) / 128, 128, 0, e->s>>>(P.tok, B, tc, d.vocab, e->seen, e->seen_words);
      CHECK_LAUNCH();
    }
    if ((rc = prefill_chunk(e, P, tc, e->s))) return rc;
    if (t0 + tc == T) {  // the last token of every sequence: final norm, LM head, next token
      last_rows_kernel<<<B, 256, 0, e->s>>>(P.x, tc, d.d_model, e->x);
      CHECK_LAUNCH();
      if ((rc = enqueue_head(e, e->s))) return rc;
      if (e->s_temp > 0.f &&
          (rc = dfssm_sample(e->logits, B, d.vocab, e->seen, e->s_temp, e->s_top_p, e->s_rep, e->s_seed,
                             reinterpret_cast<uint64_t*>(e->counters), e->tokens, nullptr, nullptr, e->s)))
        return rc;
    }
  }
  if (logits_dev)
    CU(cudaMemcpyAsync(logits_dev, e->logits, (size_t)B * d.vocab * 4, cudaMemcpyDeviceToDevice, e->s));
  if (next_tokens_dev) CU(cudaMemcpyAsync(next_tokens_dev, e->tokens, (size_t)B * 4, cudaMemcpyDeviceToDevice, e->s));
  CU(cudaEventRecord(e->ev_out, e->s));
  CU(cudaStreamWaitEvent(us, e->ev_out, 0));
  owner->order_s = us;
  owner->order_valid = true;
  return DFSSM_OK;
}

// A shallow copy of the engine whose per-sequence buffers start at slot `first` and whose batch is
// `count` (per-layer strides stay those of max_batch).  It runs the per-op kernels eagerly (mode 2:
// no captured graph, no persistent kernel, whose pointers are fixed to slot 0) and owns nothing:
// it is never destroyed, and prompt-row buffers come from the owning engine.
dfssm_engine slot_view(const dfssm_engine* e, int first, int count) {
  const dfssm_dims& d = e->d;
  const size_t kmax = d.d_inner > d.d_model ? d.d_inner : d.d_model, f = (size_t)first;
  dfssm_engine v = *e;
  v.ssm += f * d.nheads * DFSSM_HEADDIM * DFSSM_DSTATE;
  v.conv += f * 3 * d.d_xbc;
  v.x += f * d.d_model;
  v.xn += f * kmax;
  v.q += f * kmax;
  v.xs += f;
  v.qsum += f;
  v.t += f * kRank;
  v.proj += f * d.n_in;
  v.gated += f * d.d_inner;
  v.logits += f * d.vocab;
  v.best += f;
  v.tokens += f;
  v.seen += f * v.seen_words;
  v.counters += f;
  v.batch = count;
  v.mode = 2;
  v.gexec = nullptr;
  v.graph_batch = v.graph_mode = -1;
  v.persist = nullptr;
  return v;
}

}  // namespace

int dfssm_prefill(dfssm_engine* e, const int32_t* tokens_dev, int T, float* logits_dev, int32_t* next_tokens_dev,
                  void* stream) {
  return prefill_impl(e, e, tokens_dev, T, logits_dev, next_tokens_dev, stream);
}

int dfssm_prefill_slots(dfssm_engine* e, int first, int count, const int32_t* tokens_dev, int T, float* logits_dev,
                        int32_t* next_tokens_dev, void* stream) {
  if (!e) return dfssm_fail(DFSSM_ERR_ARG, "NULL engine");
  if (first < 0 || count < 1 || first + count > e->batch)
    return dfssm_fail(DFSSM_ERR_ARG, "slots [%d, %d) outside the batch of %d", first, first + count, e->batch);
  dfssm_engine v = slot_view(e, first, count);
  return prefill_impl(&v, e, tokens_dev, T, logits_dev, next_tokens_dev, stream);
}
