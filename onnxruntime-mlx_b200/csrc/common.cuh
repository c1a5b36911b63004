// Shared device/host helpers for the sm_100a kernels of the B200 int4 decode EP.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "status.h"

namespace b200ep {

// ONNX TensorProto element types (identical to ONNXTensorElementDataType).
enum DType : int { kF32 = 1, kU8 = 2, kI32 = 6, kI64 = 7, kF16 = 10, kBF16 = 16 };

inline int dtype_size(int dt) {
  switch (dt) {
    case kF32: case kI32: return 4;
    case kF16: case kBF16: return 2;
    case kU8: return 1;
    case kI64: return 8;
  }
  return 0;
}
inline bool is_float_dtype(int dt) { return dt == kF32 || dt == kF16 || dt == kBF16; }

template <typename T> struct Num;
template <> struct Num<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Num<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Num<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

template <typename T> __device__ __forceinline__ float to_f(T v) { return Num<T>::to_f(v); }
template <typename T> __device__ __forceinline__ T from_f(float v) { return Num<T>::from_f(v); }
// Round an fp32 value through T (identity for fp32).
template <typename T> __device__ __forceinline__ float round_through(float v) {
  return to_f<T>(from_f<T>(v));
}

// ---- PTX wrappers: mbarrier + bulk (TMA) copies -------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait on an mbarrier phase.  Returns false when the iteration limit ran out; the
// caller records an error and stops using the pipeline instead of hanging the SM.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, uint32_t max_iters = 1u << 22) {
  uint32_t done = 0;
  for (uint32_t it = 0; it < max_iters; ++it) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    if (done) return true;
  }
  return false;
}

// 1-D bulk copy global -> shared through the TMA engine; completion is signalled on `bar`
// with the byte count.  dst/src must be 16-byte aligned and bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Orders this thread's prior generic-proxy global writes before later async-proxy (TMA) reads.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Device-side error word shared by all kernels of this library: the first failing kernel
// stores its code (atomicCAS from 0); the host reads and clears it through b200ep_device_error.
struct DeviceErrorSlot {
  int code;
  int detail;
};
DeviceErrorSlot* device_error_slot();  // host: device address of the current device's slot
__device__ __forceinline__ void report_device_error(DeviceErrorSlot* slot, int code, int detail) {
  if (slot && atomicCAS(&slot->code, 0, code) == 0) slot->detail = detail;
}

inline int div_up(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// ---- programmatic dependent launch ------------------------------------------------------------
// Kernels of a decode chain are launched with programmatic stream serialization: a kernel may be
// scheduled while its predecessor is still running (its CTAs start once the predecessor's CTAs
// have all executed pdl_trigger or exited).  Every such kernel calls pdl_wait() before it touches
// memory an earlier kernel of the stream writes (and before it writes anything an earlier kernel
// reads); the wait returns once the predecessor grid has completed and its writes are visible.
// pdl_trigger() is only executed after the kernel's own pdl_wait(), so when a kernel starts, every
// kernel before its predecessor has completed: code before the wait may read data written two or
// more kernels back (weights, a KV cache row of an earlier step) but nothing the predecessor
// writes.  Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();  // false when ONNXRUNTIME_EP_B200_NO_PDL is set, or while a PdlOff lives

// Launches issued on this thread while a PdlOff is alive wait for the previous kernel of the
// stream to complete: for a kernel whose pre-wait code reads what its immediate predecessor writes
// (attention reading lengths that the integer glue just computed).
struct PdlOff {
  PdlOff();
  ~PdlOff();
  PdlOff(const PdlOff&) = delete;
  PdlOff& operator=(const PdlOff&) = delete;
};

// SMs of the current device (cached; every GPU of a node is the same part)
inline int num_sms() {
  static int sms = 0;
  if (!sms) {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    sms = n > 0 ? n : 148;
  }
  return sms;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace b200ep
