// RMS norms for sm_100a: RMSNormalization / SimplifiedLayerNormalization and
// SkipSimplifiedLayerNormalization (reference: rust/src/ops/norm.rs:163-246, which calls
// mlx_fast_rms_norm).  One CTA per row; the row is read once into registers (vectorised,
// up to 8 values per thread per pass), the sum of squares is reduced in fp32 across the CTA,
// and the scaled row is written back.  The skip form writes the fp32 sum rounded to the I/O
// dtype as the residual output and normalises the unrounded sum.
#include "../common.cuh"
#include "kernels.h"

namespace b200ep {

constexpr int kRmsThreads = 256;
constexpr int kRmsMaxPerThread = 32;  // hidden <= 8192 held in registers

template <typename T, bool SKIP>
__global__ void __launch_bounds__(kRmsThreads)
rms_norm_kernel(const T* __restrict__ X, const T* __restrict__ skip, const T* __restrict__ gamma,
                T* __restrict__ Y, T* __restrict__ R, int64_t hidden, float eps) {
  __shared__ float red[kRmsThreads / 32];
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const T* x = X + row * hidden;
  const T* sk = SKIP ? skip + row * hidden : nullptr;
  float v[kRmsMaxPerThread];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kRmsMaxPerThread; ++c) {
    const int64_t j = threadIdx.x + (int64_t)c * kRmsThreads;
    float t = 0.f;
    if (j < hidden) {
      t = to_f<T>(x[j]);
      if (SKIP) {
        t += to_f<T>(sk[j]);
        if (R) R[row * hidden + j] = from_f<T>(t);
      }
    }
    v[c] = t;
    ss = fmaf(t, t, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < kRmsThreads / 32 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)hidden + eps);
#pragma unroll
  for (int c = 0; c < kRmsMaxPerThread; ++c) {
    const int64_t j = threadIdx.x + (int64_t)c * kRmsThreads;
    if (j < hidden) Y[row * hidden + j] = from_f<T>(v[c] * inv * to_f<T>(gamma[j]));
  }
}

// The same arithmetic with 16-byte accesses (8 values) when hidden % 8 == 0 and every pointer is
// 16-byte aligned: a decode row of 4096 is two loads per thread instead of sixteen.
template <typename T, bool SKIP>
__global__ void __launch_bounds__(kRmsThreads)
rms_norm_vec_kernel(const T* __restrict__ X, const T* __restrict__ skip, const T* __restrict__ gamma,
                    T* __restrict__ Y, T* __restrict__ R, int64_t hidden, float eps) {
  constexpr int kC = kRmsThreads * kRmsMaxPerThread / (8 * kRmsThreads);  // chunks of 8 per thread
  __shared__ float red[kRmsThreads / 32];
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const int64_t nch = hidden / 8;
  const uint4* x = reinterpret_cast<const uint4*>(X + row * hidden);
  const uint4* sk = SKIP ? reinterpret_cast<const uint4*>(skip + row * hidden) : nullptr;
  uint4 xv[kC], sv[kC];
#pragma unroll
  for (int c = 0; c < kC; ++c) {
    const int64_t j = threadIdx.x + (int64_t)c * kRmsThreads;
    xv[c] = j < nch ? x[j] : make_uint4(0, 0, 0, 0);
    if (SKIP) sv[c] = j < nch ? sk[j] : make_uint4(0, 0, 0, 0);
  }
  float v[kC][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kC; ++c) {
    const T* xh = reinterpret_cast<const T*>(&xv[c]);
    const T* sh = reinterpret_cast<const T*>(&sv[c]);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float t = to_f<T>(xh[e]);
      if (SKIP) t += to_f<T>(sh[e]);
      v[c][e] = t;
      ss = fmaf(t, t, ss);
    }
    const int64_t j = threadIdx.x + (int64_t)c * kRmsThreads;
    if (SKIP && R && j < nch) {
      uint4 o;
      T* oh = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) oh[e] = from_f<T>(v[c][e]);
      reinterpret_cast<uint4*>(R + row * hidden)[j] = o;
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < kRmsThreads / 32 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)hidden + eps);
  const uint4* g = reinterpret_cast<const uint4*>(gamma);
#pragma unroll
  for (int c = 0; c < kC; ++c) {
    const int64_t j = threadIdx.x + (int64_t)c * kRmsThreads;
    if (j < nch) {
      const uint4 gv = g[j];
      const T* gh = reinterpret_cast<const T*>(&gv);
      uint4 o;
      T* oh = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) oh[e] = from_f<T>(v[c][e] * inv * to_f<T>(gh[e]));
      reinterpret_cast<uint4*>(Y + row * hidden)[j] = o;
    }
  }
}

namespace {
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename T>
cudaError_t launch_t(const RmsArgs& a, cudaStream_t st) {
  if (a.rows == 0) return cudaSuccess;
  dim3 grid((unsigned)a.rows);
  if (sizeof(T) == 2 && a.hidden % 8 == 0 && aligned16(a.X) && aligned16(a.gamma) && aligned16(a.Y) &&
      (!a.skip || aligned16(a.skip)) && (!a.residual || aligned16(a.residual))) {
    if (a.skip)
      return launch_k(rms_norm_vec_kernel<T, true>, grid, dim3(kRmsThreads), 0, st, static_cast<const T*>(a.X),
                      static_cast<const T*>(a.skip), static_cast<const T*>(a.gamma), static_cast<T*>(a.Y),
                      static_cast<T*>(a.residual), a.hidden, a.eps);
    return launch_k(rms_norm_vec_kernel<T, false>, grid, dim3(kRmsThreads), 0, st, static_cast<const T*>(a.X),
                    static_cast<const T*>(nullptr), static_cast<const T*>(a.gamma), static_cast<T*>(a.Y),
                    static_cast<T*>(nullptr), a.hidden, a.eps);
  }
  if (a.skip)
    return launch_k(rms_norm_kernel<T, true>, grid, dim3(kRmsThreads), 0, st, static_cast<const T*>(a.X),
                    static_cast<const T*>(a.skip), static_cast<const T*>(a.gamma), static_cast<T*>(a.Y),
                    static_cast<T*>(a.residual), a.hidden, a.eps);
  return launch_k(rms_norm_kernel<T, false>, grid, dim3(kRmsThreads), 0, st, static_cast<const T*>(a.X),
                  static_cast<const T*>(nullptr), static_cast<const T*>(a.gamma), static_cast<T*>(a.Y),
                  static_cast<T*>(nullptr), a.hidden, a.eps);
}
}  // namespace

cudaError_t launch_rms_norm(const RmsArgs& a, cudaStream_t st) {
  if (a.hidden > (int64_t)kRmsThreads * kRmsMaxPerThread) return cudaErrorInvalidValue;
  switch (a.dtype) {
    case kF32: return launch_t<float>(a, st);
    case kF16: return launch_t<__half>(a, st);
    case kBF16: return launch_t<__nv_bfloat16>(a, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace b200ep
