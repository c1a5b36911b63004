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
// the workspace without the optional transposed-value region of the tensor-core prompt kernel
// (a smaller workspace runs prompts on the mma.sync kernel)
size_t gqa_workspace_min_bytes(const b200ep_gqa_params& p);

// Tensor-core (tcgen05) prompt attention for head size 128 (gqa_umma.cu), launched after the
// append kernel: qrot = rotated query rows (fp32, rounded through the I/O type), vt = a workspace
// of gqa_umma_vt_bytes for the transposed value rows, lt = gqa_umma_lt(cap) keys per V^T row.
struct UmmaAttnArgs {
  const float* qrot;
  const void* kv_k;
  const void* kv_v;
  void* vt;
  const int32_t* seqlens;
  void* out;
  struct DeviceErrorSlot* err;
  int B, S, H, HK, G, cap, max_seq, do_rotary, local_window, lt, dtype;
  float scale_log2;
};
int64_t gqa_umma_lt(int64_t cap);
size_t gqa_umma_vt_bytes(int64_t batch, int64_t kv_heads, int64_t cap);
bool gqa_umma_supported(int64_t batch, int64_t kv_heads, int64_t head_size, int64_t cap, int dtype);
cudaError_t launch_gqa_umma_prefill(const UmmaAttnArgs& a, cudaStream_t st);
// Validates geometry (returns a B200EP_* status and message via set_error) and launches.
int launch_gqa(const GqaArgs& a, cudaStream_t st);

// GroupQueryAttention with sliding_window_cache = 1 (gqa_sliding.cu): past / present [B, kv_heads,
// cap, D] (they may be the same buffers), p.cap = cap, p.local_window = the window (<= cap); packed
// or separate q / k / v; no qk norm, no attention_bias.
struct GqaSlidingArgs {
  b200ep_gqa_params p;
  const void* query;
  const void* key;
  const void* value;
  const void* past_key;
  const void* past_value;
  void* present_key;
  void* present_value;
  const int32_t* seqlens_k;
  const void* cos_cache;
  const void* sin_cache;
  void* out;
  int dtype;
  void* workspace;  // gqa_sliding_workspace_bytes, zeroed before its first use
  size_t workspace_bytes;
};
size_t gqa_sliding_workspace_bytes(const b200ep_gqa_params& p, int dtype);
int launch_gqa_sliding(const GqaSlidingArgs& a, cudaStream_t st);

// PagedAttention rows (fp16 / bf16, head_size 64 / 128, at most 8 query heads per kv head, fewer
// than 65536 rows, 16-byte aligned caches) on the tensor-core decode kernel of gqa.cu; the new
// rows must already be in the caches.
struct PagedMmaArgs {
  const void* query;
  void* key_cache;
  void* value_cache;
  const int32_t* cum;
  const int32_t* past;
  const int32_t* block_table;
  const void* cos_cache;
  const void* sin_cache;
  void* out;
  int dtype, batch, num_tokens, num_heads, kv_heads, head_size;
  int num_blocks, block_size, max_blocks, max_seq, rotary_half, do_rotary, interleaved;
  float scale;
};
cudaError_t launch_paged_mma(const PagedMmaArgs& a, cudaStream_t st);
// Prompt chunks (the same conditions) on the tensor-core prefill kernel of gqa.cu; the rotated q
// rows (rounded to the I/O dtype) must already be in `out`.
cudaError_t launch_paged_prefill(const PagedMmaArgs& a, cudaStream_t st);

}  // namespace b200ep
