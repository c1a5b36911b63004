/*
 * b200ep.h — kernel-level C ABI of the B200 int4 decode execution provider.
 *
 * The reference EP (justinchuby/onnxruntime-mlx) hands its hot operators to the
 * MLX C API (mlx-c 0.6): mlx_quantized_matmul, mlx_fast_scaled_dot_product_attention,
 * mlx_fast_rope, mlx_slice_update and mlx_fast_rms_norm.  Each entry point below
 * replaces one of those call sites with a hand-written sm_100a kernel; the
 * comment on each names the reference call it replaces (file:line within the
 * reference project).
 *
 * Conventions
 *   - Plain pointers and sizes only.  Tensor pointers are DEVICE pointers unless
 *     stated otherwise; `stream` is a cudaStream_t (NULL = legacy default stream).
 *   - dtype arguments use ONNX TensorProto element types: 1 = float32,
 *     10 = float16, 16 = bfloat16 (2 = uint8, 6 = int32 where noted).
 *   - Every function returns B200EP_OK (0) or a non-zero status and never
 *     aborts the process; b200ep_last_error() returns the calling thread's last
 *     message.  Launches are asynchronous: faults detected inside a kernel (a
 *     sequence position outside the caches, a bounded wait that ran out) are
 *     recorded in a per-device error word read by b200ep_device_error().
 *   - No entry point synchronises the stream or allocates per call, except
 *     where a "workspace" argument is NULL (see b200ep_gqa_workspace_size).
 */
#ifndef B200EP_H_
#define B200EP_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define B200EP_API __declspec(dllexport)
#else
#define B200EP_API __attribute__((visibility("default")))
#endif

enum {
  B200EP_OK = 0,
  B200EP_EINVAL = 1,       /* invalid argument or tensor geometry */
  B200EP_ERANGE = 2,       /* sequence position / length outside the buffers */
  B200EP_ECUDA = 3,        /* CUDA runtime error */
  B200EP_ENOMEM = 4,       /* device allocation failed */
  B200EP_EUNSUPPORTED = 5, /* form the kernels do not implement (the EP does not claim it) */
  B200EP_ETIMEOUT = 6,     /* a bounded device-side wait ran out */
  B200EP_ENCCL = 7,        /* NCCL error */
  B200EP_EINTERNAL = 8
};

/* Library / device state ---------------------------------------------------------------------- */
B200EP_API int b200ep_version(void);
B200EP_API const char* b200ep_last_error(void);
/* Reads (and with clear != 0 resets) the current device's kernel error word.  *code = 0 means no
 * kernel reported a fault since the last clear.  Synchronises the device. */
B200EP_API int b200ep_device_error(int* code, int* detail, int clear);

/* MatMulNBits ---------------------------------------------------------------------------------
 * Y[M,N] = A[M,K] . W^T with W[n,k] = (q[n,k] - zp[n, k/block]) * scale[n, k/block].
 *
 * Replaces: mlx_quantized_matmul(x, w, scales, biases, transpose=true, group, bits, "affine")
 *   (rust/src/ops/quant.rs:570-601, called from matmulnbits_op quant.rs:986-1130) and the
 *   block-16 dequant + mlx_matmul fallback (quant.rs:1078-1118).
 * Layouts are ONNX Runtime's (com.microsoft MatMulNBits):
 *   A       [M, K]                         dtype
 *   B       uint8 [N, nblocks, block*bits/8]  (int4: low nibble = even k)
 *   scales  [N * nblocks]                  dtype
 *   zero_points  NULL (-> 2^(bits-1)) or uint8; int4: [N, ceil(nblocks/2)] packed, low nibble =
 *           even block; int8: [N, nblocks]
 *   Y       [M, N]                         dtype
 * bits in {4, 8}; block_size in {16, 32, 64, 128}; K need not be a multiple of block_size. */
B200EP_API int b200ep_matmulnbits(const void* A, const uint8_t* B, const void* scales,
                                  const uint8_t* zero_points, void* Y, int dtype, int64_t M,
                                  int64_t N, int64_t K, int bits, int block_size, void* stream);

/* Dequantised weight W[N, K] in out_dtype (bit-exact against (float)(q-zp)*(float)scale for
 * out_dtype float32).  Replaces the reference's cached repack + affine biases
 * (matmulnbits_repack quant.rs:634-710, matmulnbits_*_biases quant.rs:800-984). */
B200EP_API int b200ep_matmulnbits_dequant(const uint8_t* B, const void* scales,
                                          const uint8_t* zero_points, void* W, int scale_dtype,
                                          int out_dtype, int64_t N, int64_t K, int bits,
                                          int block_size, void* stream);

/* Prepacked int4 weights for the tensor-core path (fp16 / bf16 activations, bits = 4, K % 16 == 0).
 * The weight is repacked once into self-contained group records — 16 rows x 64 k of int4 values in
 * mma.sync operand order followed by that group's block scales and zero points — stored tile-major
 * so a run of rows is one contiguous stream for the TMA engine.  The B200 counterpart of the
 * reference's one-time repack to MLX words (rust/src/ops/quant.rs:634-710).
 * b200ep_matmulnbits_prepack_size gives the buffer size; b200ep_matmulnbits_prepack fills it
 * (device to device); b200ep_matmulnbits_prepacked computes Y[M,N] = A . W^T like
 * b200ep_matmulnbits (exact (q - zp) products accumulated in fp32 per block, scaled once per
 * block). */
B200EP_API int b200ep_matmulnbits_prepack_size(int64_t N, int64_t K, int bits, int block_size,
                                               size_t* bytes);
B200EP_API int b200ep_matmulnbits_prepack(const uint8_t* B, const void* scales,
                                          const uint8_t* zero_points, int dtype, int64_t N,
                                          int64_t K, int bits, int block_size, void* packed,
                                          void* stream);
B200EP_API int b200ep_matmulnbits_prepacked(const void* A, const void* packed, void* Y, int dtype,
                                            int64_t M, int64_t N, int64_t K, int bits,
                                            int block_size, void* stream);

/* RMS norms -----------------------------------------------------------------------------------
 * Y = X / sqrt(mean(X^2, last axis) + eps) * gamma, fp32 accumulation.
 * Replaces: mlx_fast_rms_norm in rms_norm_op / simplified_layer_norm_op
 *   (rust/src/ops/norm.rs:163-183). */
B200EP_API int b200ep_rms_norm(const void* X, const void* gamma, void* Y, int dtype, int64_t rows,
                               int64_t hidden, float eps, void* stream);

/* SkipSimplifiedLayerNormalization: R = X + skip; Y = rms_norm(R) * gamma; residual_out = R
 * (may be NULL).  Replaces: skip_rms_norm_op (rust/src/ops/norm.rs:229-246). */
B200EP_API int b200ep_skip_rms_norm(const void* X, const void* skip, const void* gamma, void* Y,
                                    void* residual_out, int dtype, int64_t rows, int64_t hidden,
                                    float eps, void* stream);

/* GroupQueryAttention (com.microsoft) ---------------------------------------------------------
 * Replaces the reference's GQA translation (group_query_attention_op,
 * rust/src/ops/attention.rs:556-952): mlx_fast_rope / rotate-half RoPE (attention.rs:353-495),
 * the KV append by mlx_slice_update[_dynamic] (attention.rs:534-535, 893-907) and
 * mlx_fast_scaled_dot_product_attention (attention.rs:111-135, 497-554).
 *
 * One call: RoPE on the new q/k rows at positions past_b + s, in-place append of the new k/v rows
 * into the KV buffer at [past_b, past_b + S), causal (optionally windowed / biased) attention of
 * the S query rows over keys [0, past_b + S), with past_b = seqlens_k[b] + 1 - S read from device
 * memory (so one launch configuration serves every decode step, e.g. inside a CUDA graph).
 *
 *   query   [B, S, H*D]  (packed_qkv: [B, S, (H + 2*HK)*D] and key/value NULL)
 *   key, value [B, S, HK*D]
 *   kv_key, kv_value  [B, HK, cap, D]: the shared past/present buffers, updated in place
 *   seqlens_k  int32 [B] (device)
 *   cos_cache, sin_cache  [max_seq, rotary_half] (NULL when do_rotary == 0)
 *   q_norm, k_norm  [D] per-head RMS norm weights applied before RoPE (NULL = none)
 *   attention_bias  [bias_batch (1 or B), 1, S, bias_total] additive (NULL = none)
 *   out     [B, S, H*D]
 * All float tensors share `dtype`.  The growing (non-shared) contract is served by the EP by
 * copying past into present first.  `workspace` holds split-K partials and per-(b, kv-head)
 * arrival counters; it must be zero-filled before its first use (each call leaves the counters
 * at zero again).  workspace == NULL uses a library-owned buffer allocated on first need. */
typedef struct b200ep_gqa_params {
  int64_t batch, seq, num_heads, kv_heads, head_size;
  int64_t cap;          /* axis-2 length of kv_key / kv_value */
  int64_t max_seq;      /* rows of the cos/sin caches (0 when absent) */
  int64_t rotary_half;  /* cos_cache.shape[1] */
  int32_t do_rotary, interleaved, packed_qkv;
  int32_t local_window; /* <= 0: no window */
  float scale;          /* 0 -> 1/sqrt(head_size) */
  float qk_norm_eps;
  int64_t bias_batch;   /* 0 = no attention_bias */
  int64_t bias_total;
} b200ep_gqa_params;

B200EP_API size_t b200ep_gqa_workspace_size(const b200ep_gqa_params* p);

B200EP_API int b200ep_group_query_attention(
    const b200ep_gqa_params* p, const void* query, const void* key, const void* value,
    void* kv_key, void* kv_value, const int32_t* seqlens_k, const void* cos_cache,
    const void* sin_cache, const void* q_norm, const void* k_norm, const void* attention_bias,
    void* out, int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* GroupQueryAttention with sliding_window_cache = 1 (reference: the sliding branch of
 * group_query_attention_op, rust/src/ops/attention.rs:725-880; claim 1552-1575).  past_key /
 * past_value and present_key / present_value are [batch, kv_heads, cap, head_size] (present may be
 * the past buffers themselves); p->cap is that capacity and p->local_window the window W (0 < W <=
 * cap).  After L tokens a cache holds the last end(L) rows, end(L) = L while L <= cap, else
 * L - (cap - W + 1) * ceil((L - cap) / (cap - W + 1)): rows are reclaimed from the front.  Query row
 * i of sequence b (absolute position p_b + i, p_b = seqlens_k[b] + 1 - seq) attends the W most recent
 * keys (causal window); q / k are rotated at their absolute positions; present receives the rows
 * kept after this step from row 0 and zeros after them.  Packed or separate q / k / v; no qk norm,
 * no attention_bias.  workspace: b200ep_gqa_sliding_workspace_size bytes, zero-filled before its
 * first use (null: a library-owned buffer).  Every length is read on the device. */
B200EP_API size_t b200ep_gqa_sliding_workspace_size(const b200ep_gqa_params* p, int dtype);
B200EP_API int b200ep_group_query_attention_sliding(
    const b200ep_gqa_params* p, const void* query, const void* key, const void* value, const void* past_key,
    const void* past_value, void* present_key, void* present_value, const int32_t* seqlens_k,
    const void* cos_cache, const void* sin_cache, void* out, int dtype, void* workspace, size_t workspace_bytes,
    void* stream);

/* GroupQueryAttention that allocates nothing.  No counterpart in the reference: it exists for
 * callers that may not allocate device memory once running (a server that reserves its HBM
 * budget up front and treats later cudaMalloc as failure; a decode loop that must not allocate or
 * free between tokens).  Same arguments and results as b200ep_group_query_attention without the
 * workspace: the split-K scratch is a fixed library-owned device array of
 * b200ep_gqa_noalloc_max_workspace() bytes (4 MiB) per GPU, held until the process exits.
 * Geometries whose scratch (b200ep_gqa_workspace_size) exceeds it fail with B200EP_ERANGE.  The
 * first call on a device looks up the array's address (make it before any stream capture).
 * Every call shares the array: calls whose launches overlap on the GPU race on it. */
B200EP_API int b200ep_group_query_attention_noalloc(
    const b200ep_gqa_params* p, const void* query, const void* key, const void* value,
    void* kv_key, void* kv_value, const int32_t* seqlens_k, const void* cos_cache,
    const void* sin_cache, const void* q_norm, const void* k_norm, const void* attention_bias,
    void* out, int dtype, void* stream);
B200EP_API size_t b200ep_gqa_noalloc_max_workspace(void);

/* PagedAttention (com.microsoft; reference: paged_attention_op, rust/src/ops/attention.rs:2495-2746,
 * claim 2748-2900).  Tokens of `batch` sequences are packed row after row: sequence b owns query /
 * key / value rows [cumulative_seqlens[b], cumulative_seqlens[b + 1]) and continues after
 * past_seqlens[b] cached tokens.  Its logical position p lives in physical block
 * block_table[b * max_blocks + p / block_size] at row p % block_size of the caches
 * [num_blocks, block_size, kv_heads, head_size].  The new k (RoPE'd at positions past_b + j when
 * do_rotary) and v rows are written into their slots in place; query row j attends keys
 * 0 .. past_b + j causally (fp32 softmax, scale = attr or 1/sqrt(head_size)) and writes
 * out[num_tokens, num_heads * head_size].  Rotated q and k are rounded to the I/O dtype, as the
 * reference computes RoPE in that dtype.  The control tensors are read on the device; a slot
 * outside the caches or the block table, or a position outside the cos/sin rows, skips that
 * write (its output row is zeros) and sets the device error word.  fp16 / bf16, head_size 64 or
 * 128; separate K / V caches (the LATENT layout, slot_mapping, head_sink and q/k norms are
 * declined by the claim). */
typedef struct b200ep_paged_params {
  int32_t batch;       /* sequences: cumulative_seqlens has batch + 1 entries */
  int32_t num_tokens;  /* packed rows (= cumulative_seqlens[batch]) */
  int32_t num_heads, kv_heads, head_size;
  int32_t num_blocks, block_size, max_blocks; /* caches' blocks, rows per block; block_table row */
  int32_t max_seq, rotary_half;               /* cos/sin cache rows and columns (do_rotary) */
  int32_t do_rotary, interleaved;
  float scale;                                /* 0: 1/sqrt(head_size) */
} b200ep_paged_params;
B200EP_API int b200ep_paged_attention(const b200ep_paged_params* p, const void* query, const void* key,
                                      const void* value, void* key_cache, void* value_cache,
                                      const int32_t* cumulative_seqlens, const int32_t* past_seqlens,
                                      const int32_t* block_table, const void* cos_cache,
                                      const void* sin_cache, void* out, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200EP_H_ */
