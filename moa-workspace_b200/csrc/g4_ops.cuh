// Host-side launch interface of the decode-layer kernels (internal to the library).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "g4_common.cuh"

namespace g4 {

struct QkvArgs {
  const uint16_t* x;
  const uint8_t* q_weight;
  const uint8_t* k_weight;
  const uint8_t* v_weight;
  const uint16_t* q_scale;
  const uint16_t* k_scale;
  const uint16_t* v_scale;
  const uint16_t* input_rms;
  const uint16_t* q_rms;
  const uint16_t* k_rms;
  const int32_t* kv_offset;
  const int32_t* rope_offset;
  const uint16_t* cos;
  const uint16_t* sin;
  uint16_t* k_cache;
  uint16_t* v_cache;
  uint16_t* q_out;
  int ring_len;
  int rope_rows;
};

struct AttnArgs {
  const uint16_t* q;
  const uint16_t* k_cache;
  const uint16_t* v_cache;
  const float* mask;
  uint16_t* out;
  int ring_len;
  float scale;
};

struct OArgs {
  const uint16_t* x;
  const uint16_t* post_rms;
  const uint8_t* o_weight;
  const uint16_t* o_scale;
  uint16_t* residual;
};

struct FfnArgs {
  uint16_t* residual;
  const uint16_t* pre_rms;
  const uint8_t* up_packed;
  const uint8_t* gate_packed;
  const uint8_t* down_packed;
  const uint8_t* up_scale;
  const uint8_t* gate_scale;
  const uint8_t* down_scale;
  const float* up_global;
  const float* gate_global;
  const float* down_global;
  const uint16_t* post_rms;
  const uint16_t* layer_scalar;
};

struct LaunchEnv {
  int device;
  int sm_count;
  cudaStream_t stream;
  bool pdl;  // launch with programmatic stream serialization
  Scratch sc;
};

cudaError_t prepare_proj_kernels();       // one-time attributes (dynamic shared memory)
cudaError_t prepare_attention_kernels();  // one-time attributes (clusters)
cudaError_t launch_qkv(const QkvArgs& a, const LaunchEnv& env);
cudaError_t launch_attention(const AttnArgs& a, const LaunchEnv& env);
cudaError_t launch_o(const OArgs& a, const LaunchEnv& env);
cudaError_t launch_ffn_nvfp4(const FfnArgs& a, const LaunchEnv& env);

}  // namespace g4
