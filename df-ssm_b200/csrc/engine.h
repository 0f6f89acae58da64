// Internal engine definition shared by the C-ABI and the persistent step kernel.
#pragma once
#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "../../include/dfssm.h"
#include "types.cuh"

constexpr int kMaxGroups = 4;

struct dfssm_engine {
  int device = 0;
  dfssm_dims d{};
  int emb_kind = 0;
  int max_batch = 0, batch = 0;
  int mode = 0;  // requested mode (0 = auto)
  // device memory
  char* arena = nullptr;
  size_t arena_bytes = 0;
  char* work = nullptr;
  size_t work_bytes = 0;
  std::vector<dfssm::LayerW> layers;
  dfssm::LayerW* d_layers = nullptr;  // device copy for the persistent kernel
  const int8_t* Eq = nullptr;
  const float* Es = nullptr;
  const float* norm_f = nullptr;
  float* ssm = nullptr;
  float* conv = nullptr;
  size_t ssm_layer = 0, conv_layer = 0;  // elements per layer (max_batch rows)
  __half *x = nullptr, *xn = nullptr, *xs = nullptr, *t = nullptr, *proj = nullptr, *gated = nullptr;
  int8_t* q = nullptr;
  int* qsum = nullptr;
  float* logits = nullptr;
  unsigned long long* best = nullptr;
  int* tokens = nullptr;
  unsigned int* sync = nullptr;  // persistent-kernel words: exit count, error, tag epoch
  unsigned long long* xch = nullptr;  // persistent-kernel tagged exchange words
  // sampling epilogue (dfssm_set_sampling); temperature <= 0 = greedy argmax
  float s_temp = 0.f, s_top_p = 1.f, s_rep = 1.f;
  unsigned long long s_seed = 0;
  uint32_t* seen = nullptr;               // [max_batch][seen_words] tokens already in each sequence
  int seen_words = 0;
  unsigned long long* counters = nullptr;  // [max_batch] draws so far
  int* uacc = nullptr;          // split-K scratch of the tcgen05 projection [max_batch][max(n_in, d_model)]
  unsigned* ucnt = nullptr;     // its per-tile counters
  // prompt prefill rows (dfssm_prefill), grown on demand
  char* pf = nullptr;
  size_t pf_bytes = 0;
  // execution
  cudaStream_t s = nullptr;
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;
  // The caller stream into which all of the engine's work so far is ordered (every call ends with its
  // stream waiting for the engine's work).  A persistent step on that same stream launches on it
  // directly; a call on another stream first makes the engine stream wait for it (ev_cat).
  cudaStream_t order_s = nullptr;
  bool order_valid = false;
  cudaEvent_t ev_cat = nullptr;
  cudaStream_t gs[kMaxGroups] = {};           // streams of sequence groups 1.. (group 0 uses s)
  cudaEvent_t ev_fork = nullptr, ev_join[kMaxGroups] = {};
  cudaGraphExec_t gexec = nullptr;
  int graph_batch = -1, graph_mode = -1;
  int sm_count = 148;
  void* persist = nullptr;  // persistent-kernel launch state (persistent.cu)
};

// Sets the thread's last-error message and returns `code`.
int dfssm_fail(int code, const char* fmt, ...);

// Persistent whole-step kernel (persistent.cu).
int persistent_init(dfssm_engine* e);
size_t persistent_xch_words(const dfssm_dims& d);  // tagged exchange words per replica
size_t persistent_xch_bytes(const dfssm_dims& d);  // whole exchange region (all replicas)
void persistent_destroy(dfssm_engine* e);
bool persistent_supported(const dfssm_engine* e);
int launch_persistent_step(dfssm_engine* e, cudaStream_t s);
size_t persistent_trace_entries(const dfssm_engine* e);
int launch_persistent_traced(dfssm_engine* e, unsigned long long* trace_dev, cudaStream_t s);
int launch_persistent_layers(dfssm_engine* e, int l0, int l1, int from_x, int do_head, cudaStream_t s);
int persistent_debug_skew(dfssm_engine* e);
int persistent_debug_wait_limit(dfssm_engine* e, unsigned polls);
