// Integer glue of exported decoders, run on the device when its inputs are device data: the
// attention mask -> seqlens_k chain (ReduceSum over the mask's key axis, Sub, Cast) and the
// Gather / Unsqueeze / Squeeze / Reshape copies around it.  Values known on the host (shapes,
// constants, host-resident scalars) never reach these kernels: the plan evaluates them on the host.
//   ReduceSum: rust/src/ops/reduction.rs:894 (integer sum over one axis, keepdims)
//   Add / Sub / Mul on int32 / int64: rust/src/ops/elementwise.rs:925-985 (exact integer arithmetic)
//   Cast int32 <-> int64: truncation / sign extension as ONNX Cast
//   Gather with constant indices: rust/src/ops/shape.rs:119-131 (negative indices wrap)
#include "../common.cuh"
#include "elementwise.h"

namespace b200ep {

template <typename T>
__global__ void binary_int_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ y,
                                  BinaryGeom g, int op) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < g.total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, ia = 0, ib = 0;
    for (int d = g.rank - 1; d >= 0; --d) {
      const int64_t c = rem % g.out_dims[d];
      rem /= g.out_dims[d];
      ia += c * g.a_strides[d];
      ib += c * g.b_strides[d];
    }
    const T x = a[ia], z = b[ib];
    y[i] = op == kOpAdd ? (T)(x + z) : op == kOpSub ? (T)(x - z) : (T)(x * z);
  }
}

template <typename TI, typename TO>
__global__ void cast_int_kernel(const TI* __restrict__ x, TO* __restrict__ y, int64_t n) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = (TO)x[i];
}

// One CTA per row (grid-stride over rows); the row length comes from *len_dev when given (a key
// axis whose extent changes every decode step without changing the compiled program).
template <typename TI, typename TO>
__global__ void reduce_rows_kernel(const TI* __restrict__ x, TO* __restrict__ y, int64_t rows, int64_t len,
                                   const int64_t* __restrict__ len_dev) {
  pdl_wait();
  pdl_trigger();
  __shared__ long long part[32];
  const int64_t n = len_dev ? *len_dev : len;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    long long s = 0;
    for (int64_t t = threadIdx.x; t < n; t += blockDim.x) s += (long long)x[r * n + t];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
      long long tot = 0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += part[w];
      y[r] = (TO)tot;
    }
    __syncthreads();
  }
}

// y[i] = x[idx[i]] over a 1-D integer vector; indices already normalised on the host
template <typename T>
__global__ void gather_idx_kernel(const T* __restrict__ x, T* __restrict__ y, IdxList idx) {
  pdl_wait();
  pdl_trigger();
  for (int i = threadIdx.x; i < idx.n; i += blockDim.x) y[i] = x[idx.v[i]];
}

__global__ void copy_bytes_kernel(const uint8_t* __restrict__ x, uint8_t* __restrict__ y, int64_t n) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = x[i];
}

namespace {
int grid_for(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 8)); }

template <typename F>
cudaError_t by_int(int dt, F&& f) {
  switch (dt) {
    case kI32: return f(int32_t{});
    case kI64: return f(int64_t{});
  }
  return cudaErrorInvalidValue;
}
}  // namespace

cudaError_t launch_binary_int(const void* a, const void* b, void* y, int dtype, const BinaryGeom& g, int op,
                              cudaStream_t st) {
  if (g.total == 0) return cudaSuccess;
  return by_int(dtype, [&](auto tag) {
    using T = decltype(tag);
    return launch_k(binary_int_kernel<T>, dim3(grid_for(g.total)), dim3(256), 0, st, static_cast<const T*>(a),
                    static_cast<const T*>(b), static_cast<T*>(y), g, op);
  });
}

cudaError_t launch_cast_int(const void* x, int in_dt, void* y, int out_dt, int64_t n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  return by_int(in_dt, [&](auto ti) {
    using TI = decltype(ti);
    return by_int(out_dt, [&](auto to) {
      using TO = decltype(to);
      return launch_k(cast_int_kernel<TI, TO>, dim3(grid_for(n)), dim3(256), 0, st, static_cast<const TI*>(x),
                      static_cast<TO*>(y), n);
    });
  });
}

cudaError_t launch_reduce_sum_rows(const void* x, int x_dt, void* y, int y_dt, int64_t rows, int64_t len,
                                   const int64_t* len_dev, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  return by_int(x_dt, [&](auto ti) {
    using TI = decltype(ti);
    return by_int(y_dt, [&](auto to) {
      using TO = decltype(to);
      const int grid = (int)std::min<int64_t>(rows, 148 * 8);
      return launch_k(reduce_rows_kernel<TI, TO>, dim3(grid), dim3(256), 0, st, static_cast<const TI*>(x),
                      static_cast<TO*>(y), rows, len, len_dev);
    });
  });
}

cudaError_t launch_gather_idx(const void* x, void* y, int dtype, const IdxList& idx, cudaStream_t st) {
  if (idx.n == 0) return cudaSuccess;
  return by_int(dtype, [&](auto tag) {
    using T = decltype(tag);
    return launch_k(gather_idx_kernel<T>, dim3(1), dim3(64), 0, st, static_cast<const T*>(x), static_cast<T*>(y),
                    idx);
  });
}

cudaError_t launch_copy_bytes(const void* x, void* y, int64_t bytes, cudaStream_t st) {
  if (bytes == 0) return cudaSuccess;
  return launch_k(copy_bytes_kernel, dim3(grid_for(bytes)), dim3(256), 0, st, static_cast<const uint8_t*>(x),
                  static_cast<uint8_t*>(y), bytes);
}

}  // namespace b200ep
