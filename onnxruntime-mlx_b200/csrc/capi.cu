#include <cstdlib>
// extern "C" kernel entry points declared in include/b200ep.h: argument validation, error
// reporting and the library-owned GQA workspace.  Every entry point catches C++ exceptions and
// returns a status; nothing here aborts the host process (the reference's FFI panic guard,
// rust/src/lib.rs:37-71, serves the same purpose).
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "common.cuh"
#include "kernels/kernels.h"
#include "kernels/mnb_mma.h"

namespace b200ep {

namespace {
thread_local std::string g_last_error;

// The per-device kernel error word.  Kernels get its device address from device_error_slot();
// host code never dereferences the symbol itself.
__device__ DeviceErrorSlot g_error_slot;

std::mutex g_mu;
std::unordered_map<int, DeviceErrorSlot*> g_slot_addr;  // device -> address of g_error_slot
struct Workspace {
  void* ptr = nullptr;
  size_t bytes = 0;
};
std::unordered_map<int, Workspace> g_gqa_ws;  // device -> library-owned GQA workspace
}  // namespace

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}
void clear_error() { g_last_error.clear(); }

DeviceErrorSlot* device_error_slot() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_slot_addr.find(dev);
  if (it != g_slot_addr.end()) return it->second;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_error_slot) != cudaSuccess) return nullptr;
  g_slot_addr[dev] = static_cast<DeviceErrorSlot*>(p);
  return static_cast<DeviceErrorSlot*>(p);
}

// Library-owned GQA workspace for callers that pass none: grown on demand, zero-filled.
static int library_gqa_workspace(size_t bytes, cudaStream_t st, void** out) {
  int dev = 0;
  B200EP_CUDA_RET(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_mu);
  Workspace& w = g_gqa_ws[dev];
  if (w.bytes < bytes) {
    if (w.ptr) {
      B200EP_CUDA_RET(cudaStreamSynchronize(st));
      cudaFree(w.ptr);
      w.ptr = nullptr;
      w.bytes = 0;
    }
    if (cudaMalloc(&w.ptr, bytes) != cudaSuccess) {
      cudaGetLastError();
      return set_error(B200EP_ENOMEM, "GroupQueryAttention: workspace allocation failed");
    }
    B200EP_CUDA_RET(cudaMemsetAsync(w.ptr, 0, bytes, st));
    w.bytes = bytes;
  }
  *out = w.ptr;
  return B200EP_OK;
}

static int check_mnb_common(int64_t N, int64_t K, int bits, int block) {
  B200EP_CHECK_ARG(N > 0 && K > 0, "MatMulNBits: N and K must be > 0");
  B200EP_CHECK_ARG(bits == 4 || bits == 8, "MatMulNBits: only 4-bit and 8-bit weights are supported");
  B200EP_CHECK_ARG(block == 16 || block == 32 || block == 64 || block == 128,
                   "MatMulNBits: block_size must be 16, 32, 64, or 128");
  B200EP_CHECK_ARG(N < (1ll << 31) && K < (1ll << 31), "MatMulNBits: N and K must be < 2^31");
  return B200EP_OK;
}

}  // namespace b200ep

using namespace b200ep;

#define B200EP_GUARD_BEGIN try {
#define B200EP_GUARD_END                                                    \
  }                                                                         \
  catch (const std::exception& e) {                                         \
    return set_error(B200EP_EINTERNAL, std::string("exception: ") + e.what()); \
  }                                                                         \
  catch (...) {                                                             \
    return set_error(B200EP_EINTERNAL, "unknown exception");                \
  }

namespace b200ep {
namespace {
thread_local int t_pdl_off = 0;
}
PdlOff::PdlOff() { ++t_pdl_off; }
PdlOff::~PdlOff() { --t_pdl_off; }
bool pdl_enabled() {
  static const bool on = getenv("ONNXRUNTIME_EP_B200_NO_PDL") == nullptr;
  return on && t_pdl_off == 0;
}
}  // namespace b200ep

extern "C" {

B200EP_API int b200ep_version(void) { return 10000; }

B200EP_API const char* b200ep_last_error(void) { return g_last_error.c_str(); }

B200EP_API int b200ep_device_error(int* code, int* detail, int clear) {
  B200EP_GUARD_BEGIN
  DeviceErrorSlot* slot = device_error_slot();
  if (!slot) return set_error(B200EP_ECUDA, "device error slot unavailable");
  B200EP_CUDA_RET(cudaDeviceSynchronize());
  DeviceErrorSlot h{};
  B200EP_CUDA_RET(cudaMemcpy(&h, slot, sizeof(h), cudaMemcpyDeviceToHost));
  if (code) *code = h.code;
  if (detail) *detail = h.detail;
  if (clear) B200EP_CUDA_RET(cudaMemset(slot, 0, sizeof(h)));
  return B200EP_OK;
  B200EP_GUARD_END
}

B200EP_API int b200ep_matmulnbits(const void* A, const uint8_t* B, const void* scales,
                                  const uint8_t* zero_points, void* Y, int dtype, int64_t M,
                                  int64_t N, int64_t K, int bits, int block_size, void* stream) {
  B200EP_GUARD_BEGIN
  int rc = check_mnb_common(N, K, bits, block_size);
  if (rc) return rc;
  B200EP_CHECK_ARG(is_float_dtype(dtype), "MatMulNBits: A, scales and Y must be float32/float16/bfloat16");
  B200EP_CHECK_ARG(M >= 0 && M < (1ll << 31), "MatMulNBits: bad M");
  B200EP_CHECK_ARG(M == 0 || (A && B && scales && Y), "MatMulNBits: null tensor pointer");
  MnbArgs a{A, B, scales, zero_points, Y, dtype, M, N, K, bits, block_size};
  return cuda_status(launch_matmulnbits(a, static_cast<cudaStream_t>(stream)), "MatMulNBits launch");
  B200EP_GUARD_END
}

B200EP_API int b200ep_matmulnbits_dequant(const uint8_t* B, const void* scales,
                                          const uint8_t* zero_points, void* W, int scale_dtype,
                                          int out_dtype, int64_t N, int64_t K, int bits,
                                          int block_size, void* stream) {
  B200EP_GUARD_BEGIN
  int rc = check_mnb_common(N, K, bits, block_size);
  if (rc) return rc;
  B200EP_CHECK_ARG(is_float_dtype(scale_dtype) && is_float_dtype(out_dtype),
                   "MatMulNBits dequant: dtypes must be float32/float16/bfloat16");
  B200EP_CHECK_ARG(B && scales && W, "MatMulNBits dequant: null tensor pointer");
  MnbDequantArgs a{B, scales, zero_points, W, scale_dtype, out_dtype, N, K, bits, block_size};
  return cuda_status(launch_matmulnbits_dequant(a, static_cast<cudaStream_t>(stream)),
                     "MatMulNBits dequant launch");
  B200EP_GUARD_END
}

static int packed_args(int64_t N, int64_t K, int bits, int block, int dtype, MnbPacked* p) {
  int rc = check_mnb_common(N, K, bits, block);
  if (rc) return rc;
  B200EP_CHECK_ARG(mnb_mma_supported(dtype, bits, block, K),
                   "MatMulNBits prepacked path needs fp16/bf16, bits = 4 and K % 16 == 0");
  *p = mnb_packed_geometry(N, K, block);
  return B200EP_OK;
}

B200EP_API int b200ep_matmulnbits_prepack_size(int64_t N, int64_t K, int bits, int block_size, size_t* bytes) {
  B200EP_GUARD_BEGIN
  int rc = check_mnb_common(N, K, bits, block_size);
  if (rc) return rc;
  B200EP_CHECK_ARG(bits == 4 && K % 16 == 0, "MatMulNBits prepacked path needs bits = 4 and K % 16 == 0");
  if (bytes) *bytes = mnb_packed_geometry(N, K, block_size).bytes;
  return B200EP_OK;
  B200EP_GUARD_END
}

B200EP_API int b200ep_matmulnbits_prepack(const uint8_t* B, const void* scales, const uint8_t* zero_points,
                                          int dtype, int64_t N, int64_t K, int bits, int block_size, void* packed,
                                          void* stream) {
  B200EP_GUARD_BEGIN
  MnbPacked p;
  int rc = packed_args(N, K, bits, block_size, dtype, &p);
  if (rc) return rc;
  B200EP_CHECK_ARG(B && scales && packed, "MatMulNBits prepack: null pointer");
  p.w = packed;
  return cuda_status(launch_mnb_prepack(B, scales, zero_points, dtype, p, static_cast<cudaStream_t>(stream)),
                     "MatMulNBits prepack launch");
  B200EP_GUARD_END
}

B200EP_API int b200ep_matmulnbits_prepacked(const void* A, const void* packed, void* Y, int dtype, int64_t M,
                                            int64_t N, int64_t K, int bits, int block_size, void* stream) {
  B200EP_GUARD_BEGIN
  MnbPacked p;
  int rc = packed_args(N, K, bits, block_size, dtype, &p);
  if (rc) return rc;
  B200EP_CHECK_ARG(M >= 0 && M < (1ll << 31), "MatMulNBits: bad M");
  B200EP_CHECK_ARG(M == 0 || (A && packed && Y), "MatMulNBits prepacked: null pointer");
  B200EP_CHECK_ARG(reinterpret_cast<uintptr_t>(packed) % 16 == 0 && reinterpret_cast<uintptr_t>(A) % 4 == 0,
                   "MatMulNBits prepacked: packed weights must be 16-byte and A 4-byte aligned");
  p.w = const_cast<void*>(packed);
  // many rows: the tcgen05 GEMM; decode-sized rows: the streaming GEMV
  if (mnb_gemm_supported(M, K, A))
    return cuda_status(launch_mnb_gemm(A, p, Y, dtype, M, static_cast<cudaStream_t>(stream)),
                       "MatMulNBits prepacked GEMM launch");
  return cuda_status(launch_mnb_packed(A, p, Y, dtype, M, static_cast<cudaStream_t>(stream)),
                     "MatMulNBits prepacked launch");
  B200EP_GUARD_END
}

static int rms_common(const void* X, const void* skip, const void* gamma, void* Y, void* residual,
                      int dtype, int64_t rows, int64_t hidden, float eps, void* stream) {
  B200EP_CHECK_ARG(is_float_dtype(dtype), "RMS norm: dtype must be float32/float16/bfloat16");
  B200EP_CHECK_ARG(rows >= 0 && hidden > 0, "RMS norm: rows >= 0 and hidden > 0 required");
  B200EP_CHECK_ARG(hidden <= 8192, "RMS norm: hidden > 8192 is not supported");
  B200EP_CHECK_ARG(rows < (1ll << 31), "RMS norm: too many rows");
  B200EP_CHECK_ARG(rows == 0 || (X && gamma && Y), "RMS norm: null tensor pointer");
  B200EP_CHECK_ARG(eps >= 0.f, "RMS norm: epsilon must be >= 0");
  RmsArgs a{X, skip, gamma, Y, residual, dtype, rows, hidden, eps};
  return cuda_status(launch_rms_norm(a, static_cast<cudaStream_t>(stream)), "RMS norm launch");
}

B200EP_API int b200ep_rms_norm(const void* X, const void* gamma, void* Y, int dtype, int64_t rows,
                               int64_t hidden, float eps, void* stream) {
  B200EP_GUARD_BEGIN
  return rms_common(X, nullptr, gamma, Y, nullptr, dtype, rows, hidden, eps, stream);
  B200EP_GUARD_END
}

B200EP_API int b200ep_skip_rms_norm(const void* X, const void* skip, const void* gamma, void* Y,
                                    void* residual_out, int dtype, int64_t rows, int64_t hidden,
                                    float eps, void* stream) {
  B200EP_GUARD_BEGIN
  B200EP_CHECK_ARG(rows == 0 || skip, "SkipSimplifiedLayerNormalization: skip is null");
  return rms_common(X, skip, gamma, Y, residual_out, dtype, rows, hidden, eps, stream);
  B200EP_GUARD_END
}

B200EP_API size_t b200ep_gqa_workspace_size(const b200ep_gqa_params* p) {
  try {
    if (!p || p->batch <= 0 || p->seq <= 0 || p->num_heads <= 0 || p->kv_heads <= 0 ||
        p->head_size <= 0 || p->num_heads % p->kv_heads)
      return 0;
    return gqa_workspace_bytes(*p);
  } catch (...) {
    return 0;
  }
}

B200EP_API int b200ep_group_query_attention(
    const b200ep_gqa_params* p, const void* query, const void* key, const void* value,
    void* kv_key, void* kv_value, const int32_t* seqlens_k, const void* cos_cache,
    const void* sin_cache, const void* q_norm, const void* k_norm, const void* attention_bias,
    void* out, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  B200EP_GUARD_BEGIN
  B200EP_CHECK_ARG(p != nullptr, "GroupQueryAttention: params is null");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GqaArgs a{*p, query, key, value, kv_key, kv_value, seqlens_k, cos_cache, sin_cache,
            q_norm, k_norm, attention_bias, out, dtype, workspace, workspace_bytes};
  if (!workspace) {
    const size_t need = b200ep_gqa_workspace_size(p);
    B200EP_CHECK_ARG(need > 0, "GroupQueryAttention: invalid geometry");
    int rc = library_gqa_workspace(need, st, &a.workspace);
    if (rc) return rc;
    a.workspace_bytes = need;
  }
  return launch_gqa(a, st);
  B200EP_GUARD_END
}

B200EP_API size_t b200ep_gqa_sliding_workspace_size(const b200ep_gqa_params* p, int dtype) {
  try {
    if (!p || p->batch <= 0 || p->seq <= 0 || p->num_heads <= 0 || p->kv_heads <= 0 ||
        p->head_size <= 0 || p->num_heads % p->kv_heads || p->cap <= 0)
      return 0;
    return gqa_sliding_workspace_bytes(*p, dtype);
  } catch (...) {
    return 0;
  }
}

B200EP_API int b200ep_group_query_attention_sliding(
    const b200ep_gqa_params* p, const void* query, const void* key, const void* value, const void* past_key,
    const void* past_value, void* present_key, void* present_value, const int32_t* seqlens_k,
    const void* cos_cache, const void* sin_cache, void* out, int dtype, void* workspace, size_t workspace_bytes,
    void* stream) {
  B200EP_GUARD_BEGIN
  B200EP_CHECK_ARG(p != nullptr, "GroupQueryAttention: params is null");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GqaSlidingArgs a{*p, query, key, value, past_key, past_value, present_key, present_value, seqlens_k,
                   cos_cache, sin_cache, out, dtype, workspace, workspace_bytes};
  if (!workspace) {
    const size_t need = b200ep_gqa_sliding_workspace_size(p, dtype);
    B200EP_CHECK_ARG(need > 0, "GroupQueryAttention: invalid geometry");
    int rc = library_gqa_workspace(need, st, &a.workspace);
    if (rc) return rc;
    a.workspace_bytes = need;
  }
  return launch_gqa_sliding(a, st);
  B200EP_GUARD_END
}

}  // extern "C"
