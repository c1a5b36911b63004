// b200ep_group_query_attention_noalloc: GroupQueryAttention whose split-K scratch lives in a
// fixed, library-owned device array instead of memory the caller or the library allocates.
//
// Some callers cannot allocate device memory once they are running: an inference server that
// reserves its whole HBM budget at start-up and treats any later cudaMalloc as a failure, or a
// latency-bound decode loop that must not allocate or free (cudaFree can synchronise the device)
// between tokens.  This entry point serves them: it calls no cudaMalloc, cudaFree or allocating
// library routine.  Its scratch is `g_noalloc_scratch` below, kNoAllocScratchBytes (4 MiB) per
// device, held by every GPU that loads the library until the process exits.
//
// Host code never uses the symbol itself as an address: on the first call on a device (with that
// device current) the address is looked up once with cudaGetSymbolAddress and cached.  That first
// call should therefore come before any stream capture.  Every call shares the one array: calls
// whose launches overlap on the GPU (different streams, or concurrent host threads) race on it.
// The arrival counters that must start at zero are cleared on the caller's stream at each call.
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels/kernels.h"

namespace b200ep {
namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

int noalloc_scratch(void** out) {
  int dev = 0;
  B200EP_CUDA_RET(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(B200EP_EINVAL, "device index out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return cuda_status(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return B200EP_OK;
}

}  // namespace
}  // namespace b200ep

using namespace b200ep;

extern "C" B200EP_API size_t b200ep_gqa_noalloc_max_workspace(void) { return kNoAllocScratchBytes; }

extern "C" B200EP_API int b200ep_group_query_attention_noalloc(
    const b200ep_gqa_params* p, const void* query, const void* key, const void* value, void* kv_key,
    void* kv_value, const int32_t* seqlens_k, const void* cos_cache, const void* sin_cache, const void* q_norm,
    const void* k_norm, const void* attention_bias, void* out, int dtype, void* stream) {
  try {
    B200EP_CHECK_ARG(p != nullptr, "GroupQueryAttention (no-alloc): params is null");
    B200EP_CHECK_ARG(p->batch > 0 && p->seq > 0 && p->num_heads > 0 && p->kv_heads > 0 && p->head_size > 0 &&
                         p->num_heads % p->kv_heads == 0,
                     "GroupQueryAttention (no-alloc): invalid geometry");
    const size_t need = gqa_workspace_min_bytes(*p);
    if (need > kNoAllocScratchBytes)
      return set_error(B200EP_ERANGE, "GroupQueryAttention (no-alloc): this geometry needs " + std::to_string(need) +
                                          " bytes of scratch, above the fixed " +
                                          std::to_string(kNoAllocScratchBytes) + "-byte limit");
    void* scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the per-(batch, kv-head) arrival counters lead the workspace; start them at zero
    const size_t counters = ((size_t)p->batch * p->kv_heads * sizeof(int) + 255) & ~(size_t)255;
    B200EP_CUDA_RET(cudaMemsetAsync(scratch, 0, counters, st));
    GqaArgs a{*p, query, key, value, kv_key, kv_value, seqlens_k, cos_cache, sin_cache,
              q_norm, k_norm, attention_bias, out, dtype, scratch, kNoAllocScratchBytes};
    return launch_gqa(a, st);
  } catch (const std::exception& e) {
    return set_error(B200EP_EINTERNAL, std::string("exception: ") + e.what());
  } catch (...) {
    return set_error(B200EP_EINTERNAL, "unknown exception");
  }
}
