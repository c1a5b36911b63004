// Internal launcher interface between the extern "C" layer / EP executor and the CUDA kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../../include/b200ep.h"

namespace b200ep {

struct MnbArgs {
  const void* A;
  const uint8_t* B;
  const void* scales;
  const uint8_t* zp;  // may be null
  void* Y;
  int dtype;
  int64_t M, N, K;
  int bits, block;
};
cudaError_t launch_matmulnbits(const MnbArgs& a, cudaStream_t st);

struct MnbDequantArgs {
  const uint8_t* B;
  const void* scales;
  const uint8_t* zp;
  void* W;
  int scale_dtype, out_dtype;
  int64_t N, K;
  int bits, block;
};
cudaError_t launch_matmulnbits_dequant(const MnbDequantArgs& a, cudaStream_t st);

struct RmsArgs {
  const void* X;
  const void* skip;   // null for plain RMS norm
  const void* gamma;
  void* Y;
  void* residual;     // null: not written
  int dtype;
  int64_t rows, hidden;
  float eps;
};
cudaError_t launch_rms_norm(const RmsArgs& a, cudaStream_t st);

struct GqaArgs {
  b200ep_gqa_params p;
  const void* query;
  const void* key;
  const void* value;
  void* kv_key;
  void* kv_value;
  const int32_t* seqlens_k;
  const void* cos_cache;
  const void* sin_cache;
  const void* q_norm;
  const void* k_norm;
  const void* bias;
  void* out;
  int dtype;
  void* workspace;
  size_t workspace_bytes;
};
size_t gqa_workspace_bytes(const b200ep_gqa_params& p);
// Validates geometry (returns a B200EP_* status and message via set_error) and launches.
int launch_gqa(const GqaArgs& a, cudaStream_t st);

}  // namespace b200ep
