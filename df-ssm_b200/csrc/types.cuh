// Device-side weight descriptors shared by all kernels and the host engine.
#pragma once
#include "common.cuh"

namespace dfssm {

struct ProjW {
  const uint32_t* bits;  // [N][K/32] packed signs (bit b of word j <-> column 32j+b)
  const __half* scale;   // [N]
  const __half* A16;     // [N][16] LoRA A dequantised at load: fp16(lora_A[n][r] * lora_A_scale[n])
  const __half* B16;     // [16][K] LoRA B dequantised at load: fp16(lora_B[r][k] * lora_B_scale[r])
  int N, K;
};

struct LayerW {
  ProjW in, out;
  const __half* conv_w;   // [d_xbc][4]
  const __half* conv_b;   // [d_xbc]
  const float* A_log;     // [nheads]
  const float* Dp;        // [nheads]
  const float* dt_bias;   // [nheads]
  const float* norm_w;    // [d_inner]
  const float* ln_w;      // [d_model]
};

}  // namespace dfssm
