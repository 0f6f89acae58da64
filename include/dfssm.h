/*
 * dfssm.h — C ABI of the B200 (sm_100a) DF-SSM per-token decode engine (libdfssm.so).
 *
 * Plain C: pointers, sizes and int status codes only.  Streams are passed as `void*`
 * holding a cudaStream_t (NULL = the legacy default stream).  Device pointers are
 * CUDA device addresses on the engine's device.  Every call returns DFSSM_OK (0) or a
 * dfssm_status code; dfssm_last_error() gives a message for the calling thread.
 *
 * Reference interfaces replaced (cs-cmyk/df-ssm):
 *   engine lifecycle   inference/gpu/df_ssm_inference.py:47-139  DFSSMModel.__init__/_load/_alloc_state/reset_state
 *   decode step        inference/gpu/df_ssm_inference.py:160-224  _run_layers + graph replay + LM head (forward)
 *   conv step          inference/gpu/df_ssm_kernels.cu:109-125     conv_step (pybind)
 *   SSM step           inference/gpu/df_ssm_kernels.cu:127-151     ssm_step (pybind)
 *   scaffold matmul    inference/gpu/df_ssm_inference.py:154-158  _scaffold_matmul (torch._int_mm)
 *   LM head + argmax   inference/gpu/df_ssm_inference.py:224,236  norm_out @ embedding.T, argmax
 */
#ifndef DFSSM_H
#define DFSSM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum dfssm_status {
  DFSSM_OK = 0,
  DFSSM_ERR_ARG = 1,         /* bad argument (null pointer, size out of range, ...) */
  DFSSM_ERR_FORMAT = 2,      /* malformed or truncated .dfssm image */
  DFSSM_ERR_UNSUPPORTED = 3, /* dims this build has no kernel for */
  DFSSM_ERR_CUDA = 4,        /* a CUDA runtime call failed (message has the cudaError_t) */
  DFSSM_ERR_OOM = 5,         /* device allocation failed */
  DFSSM_ERR_STATE = 6,       /* call not valid in the engine's current state */
  DFSSM_ERR_NUMERIC = 7      /* non-finite logits detected (dfssm_check_finite) */
} dfssm_status;

/* Model dimensions, all read from the .dfssm header (export_dfssm.py:106-119). */
typedef struct dfssm_dims {
  int32_t n_layer, d_model, d_inner, d_state, nheads, headdim, ngroups, vocab;
  int32_t d_xbc; /* d_inner + 2 * ngroups * d_state */
  int32_t n_in;  /* in_proj rows: 2 * d_inner + 2 * ngroups * d_state + nheads */
} dfssm_dims;

typedef struct dfssm_engine dfssm_engine;

/* Library version string. */
const char* dfssm_version(void);
/* Diagnostics (no counterpart in the reference): the binary architecture version of the library's
 * kernels as the CUDA runtime loaded them on `device` (major * 10 + minor: 100 for sm_100a). */
int dfssm_kernel_binary_version(int device, int* version);
/* Message of the last failed call on this thread ("" if none). */
const char* dfssm_last_error(void);

/* Create an engine from a .dfssm image in host memory (exporter byte map,
 * export_dfssm.py:104-193; fp16 or int8 tied embedding).  Uploads all weights to
 * `device` and allocates fp32 state for `max_batch` sequences.
 * Replaces DFSSMModel.__init__ / _load / _alloc_state (df_ssm_inference.py:48-135). */
int dfssm_create_from_memory(const void* image, size_t image_bytes, int device, int max_batch,
                             dfssm_engine** out);
/* Same, reading the image from a file path. */
int dfssm_create_from_file(const char* path, int device, int max_batch, dfssm_engine** out);
void dfssm_destroy(dfssm_engine* e);

int dfssm_get_dims(const dfssm_engine* e, dfssm_dims* out);
/* Number of sequences decoded by dfssm_step (1..max_batch).  Drops the captured graph. */
int dfssm_set_batch(dfssm_engine* e, int batch);
/* Step execution mode: 0 = automatic (3 where supported, else 1), 1 = per-op kernels replayed from a CUDA graph,
 * 2 = per-op kernels launched eagerly, 3 = persistent whole-step kernel (batch <= 8, one launch per group of up to
 * four sequences: groups of 4, then the rest; d_model and d_inner multiples of 512). */
int dfssm_set_mode(dfssm_engine* e, int mode);
int dfssm_get_mode(const dfssm_engine* e, int* mode);

/* Zero all SSM and conv state (DFSSMModel.reset_state, df_ssm_inference.py:137-139). */
int dfssm_reset(dfssm_engine* e, void* stream);

/* Zero the SSM and conv state of sequence slots [first, first + count) only, so that a finished
 * sequence's slot can take a new sequence while the others keep decoding (continuous batching).
 * The reference has no per-sequence reset (reset_state, df_ssm_inference.py:137-139, clears all). */
int dfssm_reset_slots(dfssm_engine* e, int first, int count, void* stream);

/* One decode step for the current batch: embeds tokens_dev[b] (int32 [batch], or the
 * engine's own next-token buffer when NULL, i.e. greedy continuation), runs all layers,
 * the final norm, the LM head and the greedy argmax.  Optional outputs: logits_dev
 * (fp32 [batch][vocab]; fp32 scale*int8-dot logits) and next_tokens_dev (int32 [batch]).
 * Stream-ordered; no host synchronisation and no allocation.  Calls on different streams are ordered
 * after each other by the engine (the stream of the previous call must still exist when a call on
 * another stream is made); persistent-mode steps on the previous call's stream launch on it directly.
 * Replaces DFSSMModel.forward + argmax (df_ssm_inference.py:219-224,236). */
int dfssm_step(dfssm_engine* e, const int32_t* tokens_dev, float* logits_dev,
               int32_t* next_tokens_dev, void* stream);
/* Same with host buffers: copies tokens in and next tokens / logits out (pinned or
 * pageable host memory) around the step, and synchronises the stream. */
int dfssm_step_host(dfssm_engine* e, const int32_t* tokens_host, float* logits_host,
                    int32_t* next_tokens_host, void* stream);
/* Returns DFSSM_ERR_NUMERIC when any logit of the last step is NaN/inf (synchronises). */
int dfssm_check_finite(dfssm_engine* e, void* stream);

/* Device pointers to layer `layer`'s state: ssm fp32 [max_batch][nheads][headdim][d_state]
 * and conv fp32 [max_batch][3][d_xbc] (tap-major: tap 0 is the oldest input).
 * The reference keeps these as per-layer lists h_states / conv_states
 * (df_ssm_inference.py:112-121, fp16, conv layout [B][D_XBC][3]). */
int dfssm_state_ptrs(dfssm_engine* e, int layer, float** ssm, float** conv);

/* Named internal device buffers for tests and tools: "x" (fp16 [B][d_model] residual),
 * "proj" (fp16 [B][n_in]: z | conv'd xBC | raw dt), "gated" (fp16 [B][d_inner]),
 * "logits" (fp32 [B][vocab]), "tokens" (int32 [B]); "q" (int8 [B][K] quantised activations of the
 * last per-op projection prologue, columns in the GEMV's permuted order) and "xs" (fp16 [B], their
 * scales). */
int dfssm_get_buffer(dfssm_engine* e, const char* name, void** ptr, size_t* bytes);
/* Device pointer and size of one resident weight array (read-only views; the reference exposes its
 * weights as DFSSMModel.embedding and DFSSMModel.layers, df_ssm_inference.py:51,62-110).  layer >= 0:
 * "in_bits" / "out_bits" (packed signs uint32 [N][K/32], the file's layout, where the reference keeps
 * the unpacked int8 transpose in_w_T / out_w_T), "in_scale" / "out_scale" (fp16 [N]), "in_lora_A" /
 * "out_lora_A" (fp16 [N][16]) and "in_lora_B" / "out_lora_B" (fp16 [16][K]) dequantised as the
 * reference loader does, "conv_w" (fp16 [d_xbc][4]), "conv_b" (fp16 [d_xbc]), "A_log", "D", "dt_bias"
 * (fp32 [nheads]), "norm_w" (fp32 [d_inner]), "ln_w" (fp32 [d_model]).  layer = -1: "emb_q" (int8
 * [vocab][d_model]) and "emb_s" (fp32 [vocab]) of the tied embedding, "norm_f" (fp32 [d_model]). */
int dfssm_weight_ptr(dfssm_engine* e, int layer, const char* name, void** ptr, size_t* bytes);
/* Run layer `layer` alone on the engine's "x" buffer with the kernels of the current mode
 * (per-op kernels, or the persistent kernel over the single layer when mode 3 is selected). */
int dfssm_layer_step(dfssm_engine* e, int layer, void* stream);

/* Diagnostics (no counterpart in the reference, which has no profiler hooks): number of
 * uint64 entries of a persistent-step trace, and one persistent decode step (mode 3, batch 1 to 4:
 * one launch; DFSSM_ERR_UNSUPPORTED for other batches)
 * that records %globaltimer stamps at its phase boundaries into trace_dev
 * [sm_count][4 + 16 * n_layer]: [0] start, [1] end, [2 + 16l + k] layer l point k
 * (0 alpha entry, 1 after receiving x, 3 after norm/quant/LoRA, 4 after the weight ring wait,
 *  12 after the in_proj dot products, 2 after the LoRA-t wait, 5 after the in_proj epilogue,
 *  6 after receiving B/C, 7 after the SSM, 8 before the gated exchange, 9 after receiving the
 *  gated vector, 10 after the beta norm/quant/LoRA, 13 after the out_proj dot products, 11
 *  after the LoRA-t wait and the out_proj epilogue; 14 / 15: the copy warp issued the first /
 *  last part of this layer's ring stage, 0 for the first ring-depth layers);
 * [2 + 16 n_layer] head entry, [3 + 16 n_layer] after receiving the final x. */
size_t dfssm_trace_entries(const dfssm_engine* e);
int dfssm_trace_step(dfssm_engine* e, unsigned long long* trace_dev, void* stream);

/* Test hooks of the persistent kernel's bounded waits (no counterpart in the reference).
 * dfssm_debug_set_wait_limit: polls after which every bounded wait of the persistent kernel gives up
 * and sets the error word (0 restores the default, 2^22); it applies to every engine on e's device.
 * dfssm_debug_skew_next_step: the next persistent launch runs its first CTA with the following
 * step's exchange tags, so the exchanges with it never complete: every wait runs out, the launch
 * returns, dfssm_check_finite reports DFSSM_ERR_STATE, and dfssm_reset clears the error word so
 * that later steps run normally. */
int dfssm_debug_set_wait_limit(dfssm_engine* e, unsigned polls);
int dfssm_debug_skew_next_step(dfssm_engine* e);

/* ---- stand-alone ops (reference operator replacements) ---- */

/* Scratch bytes dfssm_scaffold_gemm needs for M activation rows of length K. */
size_t dfssm_scaffold_gemm_workspace(int M, int K);
/* acc[m][n] = sum_k q[m][k] * s[n][k], s = +-1 from packed sign bits [N][K/32]
 * (bit b of word j <-> column 32j+b, 1 -> +1), q int8 row-major [M][K], acc int32 [M][N].
 * Bit-exact with torch._int_mm(q, unpack(W).T) (df_ssm_inference.py:23-29,157).
 * K % 128 == 0.  `workspace` is device memory of dfssm_scaffold_gemm_workspace(M, K) bytes. */
int dfssm_scaffold_gemm(const uint32_t* packed, const int8_t* q, int M, int N, int K,
                        int32_t* acc, void* workspace, void* stream);

/* Allocation-free variant of dfssm_scaffold_gemm (same inputs, outputs and bit-exact result),
 * for callers that cannot allocate device memory where they need the GEMM (allocator callbacks,
 * plug-in hosts that own the memory pool, loops that must not block on an allocation).  Its
 * scratch is a fixed array inside the library; it has no counterpart in the reference.
 * Limits: M * K <= 2 MiB and M <= 2048, else DFSSM_ERR_ARG.  Every GPU that loads the library
 * keeps that 2 MiB + 8 KiB array until the process exits.  The first call on each device looks
 * up the array's device address (cudaGetSymbolAddress), so make that first call before any
 * stream capture.  All calls on a device share the one array: calls that overlap on the GPU
 * (different streams, or threads racing on one device) corrupt each other's results.  Nothing
 * from a previous call is relied on; the scratch is fully rewritten every call.  Kernel choice is
 * that of dfssm_scaffold_gemm (1-bit GEMV below 8 rows, tensor-core kernels from 8 rows). */
int dfssm_scaffold_gemm_noalloc(const uint32_t* packed, const int8_t* q, int M, int N, int K,
                                int32_t* acc, void* stream);

/* Conv1d shift-register step (df_ssm_kernels.cu:27-47, conv_step): for each channel,
 * out = s0*w0 + s1*w1 + s2*w2 + x*w3 + b, state <- (s1, s2, x), xbc <- fp16(SiLU(out)).
 * conv_state fp32 [B][3][d_xbc] (tap-major), xbc fp16 [B][ld_xbc] in place,
 * conv_w fp16 [d_xbc][4], conv_b fp16 [d_xbc]. */
int dfssm_conv_step(float* conv_state, void* xbc_f16, int ld_xbc, const void* conv_w_f16,
                    const void* conv_b_f16, int batch, int d_xbc, void* stream);

/* Mamba-2 state update (df_ssm_kernels.cu:53-103, ssm_step), fp32 state:
 * xbc fp16 [B][ld_xbc] holds conv'd x [d_inner] | B [d_state] | C [d_state];
 * dt fp16 [B][ld_dt] raw (before softplus); h fp32 [B][nheads][64][128] in place;
 * y fp16 [B][ld_y] = C.h + D*x.  headdim must be 64 and d_state 128; ld_xbc % 4 == 0. */
int dfssm_ssm_step(const void* xbc_f16, int ld_xbc, const void* dt_f16, int ld_dt,
                   const float* dt_bias, const float* A_log, const float* D, float* h_state,
                   void* y_f16, int ld_y, int batch, int nheads, int headdim, int d_state,
                   void* stream);

/* RMSNorm + per-row int8 quantisation (df_ssm_inference.py:141-152, _rms_norm then
 * _quantize_to_int8) of x fp16 [batch][K] with norm weights norm_w fp32 [K]: xn fp16 [batch][K]
 * = fp16(x * rsqrt(mean(x^2) + 1e-5) * w), scale fp16 [batch] = fp16(max(amax|xn|, fp16(1e-4)) / 127)
 * and q int8 [batch][K] = clamp(rne(fp16(xn / scale))), in natural column order.  Runs the device
 * functions of the persistent step kernel's prologues.  K = 512 x {1, 2, 4, 5, 8, 10}. */
int dfssm_rmsnorm_quantize(const void* x_f16, const float* norm_w, int batch, int K, void* xn_f16, void* scale_f16,
                           int8_t* q, void* stream);

/* Scratch bytes dfssm_lm_head_argmax needs for `batch` rows. */
size_t dfssm_lm_head_workspace(int batch);
/* logits[b][v] = E_s[v] * sum_k E_q[v][k] * x[b][k] (fp32) and next[b] = argmax_v of the
 * fp16-rounded logits, first index on ties (df_ssm_inference.py:224,236 with an int8
 * embedding E_q int8 [vocab][d] and scale E_s fp32 [vocab]; x fp16 [batch][d]).
 * logits may be NULL.  d % 16 == 0. */
int dfssm_lm_head_argmax(const int8_t* E_q, const float* E_s, int vocab, int d, const void* x_f16,
                         int batch, float* logits, int32_t* next, void* workspace, void* stream);

/* Prompt prefill (replaces feeding a prompt token by token through DFSSMModel.forward,
 * df_ssm_inference.py:219-231): tokens_dev int32 [batch][T] are consumed in order, as T calls of
 * dfssm_step would, and the logits / next token after the last one are returned (either may be
 * NULL).  The projections of all batch x T token rows run as batched GEMMs and each head runs its
 * conv1d and state recurrence over the T tokens with the state in registers (chunks of 64
 * tokens), so a layer's state is read and written once per chunk.  Per token the arithmetic
 * follows the decode kernels; fp32 summation orders of the LoRA down-projection differ from the
 * batch-1 decode prologue.  Fewer than 8 rows per chunk run token by token.  Device memory for
 * the prompt rows is allocated on first use (not capturable); the state continues into
 * dfssm_step. */
int dfssm_prefill(dfssm_engine* e, const int32_t* tokens_dev, int T, float* logits_dev, int32_t* next_tokens_dev,
                  void* stream);

/* Prompt prefill of sequence slots [first, first + count) of the current batch only (continuous
 * batching: a finished sequence's slot takes a new prompt while the other slots keep their state).
 * tokens_dev int32 [count][T]; logits_dev fp32 [count][vocab] and next_tokens_dev int32 [count] (either
 * may be NULL) receive the slots' results.  The slots continue from their current state (call
 * dfssm_reset_slots first for a new sequence); the other slots' state, tokens and logits are not
 * touched.  Runs the per-op kernels of dfssm_prefill on the slots' rows (a short prompt steps token by
 * token through eagerly launched per-op kernels).  The reference has no per-slot prefill: its drivers
 * feed one prompt token per forward() for the whole batch (df_ssm_inference.py:219-231). */
int dfssm_prefill_slots(dfssm_engine* e, int first, int count, const int32_t* tokens_dev, int T, float* logits_dev,
                        int32_t* next_tokens_dev, void* stream);

/* Sampling epilogue (eval/gen_test.py:54-95, the reference's generate(): temperature,
 * repetition penalty, top-p nucleus, multinomial draw), one draw per row:
 *   l = logits / temperature;  l[v] /= rep_penalty for every v set in the row's seen bitmap;
 *   p = softmax(l);  kept = the top-p nucleus (in descending p, a token is kept while the mass
 *   ranked before it is <= top_p; tokens tied at the boundary are all kept);  next = a draw
 *   from p restricted to kept, u from splitmix64(seed, row, counters[row]), counters[row]++.
 * logits fp32 [batch][vocab]; seen_bits uint32 [batch][ceil(vocab/32)] (bit v%32 of word v/32;
 * read only); counters uint64 [batch]; next int32 [batch]; kept_mass (fraction of the
 * probability mass kept) and kept_count float/int32 [batch] may be NULL.  vocab * 4 bytes must
 * fit in one CTA's shared memory (vocab <= 57,000).  temperature and rep_penalty > 0. */
int dfssm_sample(const float* logits, int batch, int vocab, uint32_t* seen_bits, float temperature, float top_p,
                 float rep_penalty, uint64_t seed, uint64_t* counters, int32_t* next, float* kept_mass,
                 int32_t* kept_count, void* stream);
/* Switch the engine's token choice from greedy argmax to dfssm_sample (temperature <= 0 switches
 * back).  The engine keeps each sequence's seen bitmap (every token fed to dfssm_step, prompt
 * included, as the reference's ids) and draw counter; dfssm_reset / dfssm_reset_slots clear them.
 * The returned logits stay the raw fp32 logits. */
int dfssm_set_sampling(dfssm_engine* e, float temperature, float top_p, float rep_penalty, uint64_t seed);

/* Self-test (no counterpart in the reference): checks, on device `device`, the kernels'
 * two-FMA division (common.cuh div_rn_rcp, used by the activation quantiser) against IEEE fp32
 * division for every pair of finite fp16 operands with a positive divisor.  Writes the number
 * of pairs whose fp32 quotient differs to mismatch[0] and whose fp16-rounded quotient differs
 * to mismatch[1], zeros of either sign comparing equal; both must be 0.  Synchronous. */
int dfssm_selftest_division(int device, unsigned long long* mismatch);

#ifdef __cplusplus
}
#endif
#endif /* DFSSM_H */
