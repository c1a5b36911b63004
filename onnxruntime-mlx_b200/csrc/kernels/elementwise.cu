// Elementwise glue for a decoder partition (reference: rust/src/ops/elementwise.rs:925-985 —
// Add/Sub/Mul/Sigmoid/Cast) plus the fused SwiGLU produced by the plan's gate/up merge and the
// int4 GatherBlockQuantized embedding lookup (reference: rust/src/ops/quant.rs:1134-1200).
// All arithmetic in fp32, one rounding to the output dtype.
#include "../common.cuh"
#include "elementwise.h"

namespace b200ep {

template <typename T>
__global__ void binary_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ y,
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
    const float x = to_f<T>(a[ia]), z = to_f<T>(b[ib]);
    float r = op == kOpAdd ? x + z : op == kOpSub ? x - z : x * z;
    y[i] = from_f<T>(r);
  }
}

template <typename T>
__global__ void sigmoid_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = to_f<T>(x[i]);
    y[i] = from_f<T>(1.f / (1.f + __expf(-v)));
  }
}

// gu: [rows, 2n] with the gate in columns [0, n) and up in [n, 2n); h = gate * sigmoid(gate) * up
template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ gu, T* __restrict__ h, int64_t rows, int64_t n) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = rows * n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / n, c = i - r * n;
    const float g = to_f<T>(gu[r * 2 * n + c]);
    const float u = to_f<T>(gu[r * 2 * n + n + c]);
    h[i] = from_f<T>(g / (1.f + __expf(-g)) * u);
  }
}

// gu: [rows, 2n] with the gate / up columns interleaved in groups of 8 (columns 16 g .. 16 g + 7 are
// gate 8 g .. 8 g + 7, the next 8 the matching up values); h = gate * sigmoid(gate) * up
template <typename T>
__global__ void silu_mul_interleaved_kernel(const T* __restrict__ gu, T* __restrict__ h, int64_t rows, int64_t n) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = rows * n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / n, c = i - r * n;
    const int64_t src = r * 2 * n + (c >> 3) * 16 + (c & 7);
    const float g = to_f<T>(gu[src]);
    const float u = to_f<T>(gu[src + 8]);
    h[i] = from_f<T>(g / (1.f + __expf(-g)) * u);
  }
}

template <typename TI, typename TO>
__global__ void cast_kernel(const TI* __restrict__ x, TO* __restrict__ y, int64_t n) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = from_f<TO>(to_f<TI>(x[i]));
}

// one warp per gathered row; indices int32 or int64, negative indices wrap (quant.rs:1134-1200)
template <typename T, typename TI>
__global__ void gbq_kernel(const uint8_t* __restrict__ data, const T* __restrict__ scales,
                           const uint8_t* __restrict__ zp, const TI* __restrict__ idx, T* __restrict__ out,
                           int64_t n_idx, int64_t rows, int64_t dim, int block, DeviceErrorSlot* err) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= n_idx) return;
  int64_t r = (int64_t)idx[warp];
  if (r < 0) r += rows;
  if (r < 0 || r >= rows) {
    if (lane == 0) report_device_error(err, 201, (int)warp);
    return;
  }
  const int64_t nblocks = dim / block;
  const uint8_t* row = data + r * (dim / 2);
  for (int64_t j = lane; j < dim; j += 32) {
    const uint8_t byte = row[j >> 1];
    const int q = (j & 1) ? (byte >> 4) : (byte & 0x0f);
    const int64_t blk = j / block;
    int z = 8;
    if (zp) {
      const uint8_t zb = zp[r * ((nblocks + 1) / 2) + (blk >> 1)];
      z = (blk & 1) ? (zb >> 4) : (zb & 0x0f);
    }
    out[warp * dim + j] = from_f<T>((float)(q - z) * to_f<T>(scales[r * nblocks + blk]));
  }
}

// rows whose width is a multiple of 8 (and blocks of at least 8): one thread per 8 values — one
// 4-byte load of nibbles, one scale and zero point, one 16-byte (fp16 / bf16) store; grid (rows,
// dim / 2048)
template <typename T, typename TI>
__global__ void gbq8_kernel(const uint8_t* __restrict__ data, const T* __restrict__ scales,
                            const uint8_t* __restrict__ zp, const TI* __restrict__ idx, T* __restrict__ out,
                            int64_t n_idx, int64_t rows, int64_t dim, int block, DeviceErrorSlot* err) {
  pdl_wait();
  pdl_trigger();
  const int64_t w = blockIdx.x;
  const int64_t j0 = ((int64_t)blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (w >= n_idx || j0 >= dim) return;
  int64_t r = (int64_t)idx[w];
  if (r < 0) r += rows;
  if (r < 0 || r >= rows) {
    if (threadIdx.x == 0 && blockIdx.y == 0) report_device_error(err, 201, (int)w);
    return;
  }
  const int64_t nblocks = dim / block;
  const uint32_t q8 = *reinterpret_cast<const uint32_t*>(data + r * (dim / 2) + j0 / 2);
  const int64_t blk = j0 / block;
  int z = 8;
  if (zp) {
    const uint8_t zb = zp[r * ((nblocks + 1) / 2) + (blk >> 1)];
    z = (blk & 1) ? (zb >> 4) : (zb & 0x0f);
  }
  const float sc = to_f<T>(scales[r * nblocks + blk]);
  T v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = from_f<T>((float)((int)((q8 >> (4 * i)) & 15u) - z) * sc);
  if constexpr (sizeof(T) == 2) {
    *reinterpret_cast<uint4*>(out + w * dim + j0) = *reinterpret_cast<const uint4*>(v);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) out[w * dim + j0 + i] = v[i];
  }
}

namespace {
int grid_for(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 32)); }

template <typename F>
cudaError_t by_dtype(int dt, F&& f) {
  switch (dt) {
    case kF32: return f(float{});
    case kF16: return f(__half{});
    case kBF16: return f(__nv_bfloat16{});
  }
  return cudaErrorInvalidValue;
}
}  // namespace

cudaError_t launch_binary(const void* a, const void* b, void* y, int dtype, const BinaryGeom& g, int op,
                          cudaStream_t st) {
  if (g.total == 0) return cudaSuccess;
  return by_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    return launch_k(binary_kernel<T>, dim3(grid_for(g.total)), dim3(256), 0, st, static_cast<const T*>(a),
                    static_cast<const T*>(b), static_cast<T*>(y), g, op);
  });
}

cudaError_t launch_sigmoid(const void* x, void* y, int dtype, int64_t n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  return by_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    return launch_k(sigmoid_kernel<T>, dim3(grid_for(n)), dim3(256), 0, st, static_cast<const T*>(x),
                    static_cast<T*>(y), n);
  });
}

cudaError_t launch_silu_mul(const void* gu, void* h, int dtype, int64_t rows, int64_t n, cudaStream_t st) {
  if (rows * n == 0) return cudaSuccess;
  return by_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    return launch_k(silu_mul_kernel<T>, dim3(grid_for(rows * n)), dim3(256), 0, st, static_cast<const T*>(gu),
                    static_cast<T*>(h), rows, n);
  });
}

cudaError_t launch_silu_mul_interleaved(const void* gu, void* h, int dtype, int64_t rows, int64_t n,
                                        cudaStream_t st) {
  if (rows * n == 0) return cudaSuccess;
  return by_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    return launch_k(silu_mul_interleaved_kernel<T>, dim3(grid_for(rows * n)), dim3(256), 0, st,
                    static_cast<const T*>(gu), static_cast<T*>(h), rows, n);
  });
}

cudaError_t launch_cast(const void* x, int in_dt, void* y, int out_dt, int64_t n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  return by_dtype(in_dt, [&](auto ti) {
    using TI = decltype(ti);
    return by_dtype(out_dt, [&](auto to) {
      using TO = decltype(to);
      return launch_k(cast_kernel<TI, TO>, dim3(grid_for(n)), dim3(256), 0, st, static_cast<const TI*>(x),
                      static_cast<TO*>(y), n);
    });
  });
}

cudaError_t launch_gather_block_quantized(const GbqArgs& a, cudaStream_t st) {
  if (a.n_idx == 0) return cudaSuccess;
  const bool wide = a.dim % 8 == 0 && a.block % 8 == 0 && (reinterpret_cast<uintptr_t>(a.data) & 3) == 0 &&
                    (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 && a.n_idx <= 65535 * 64;
  if (wide) {
    return by_dtype(a.dtype, [&](auto tag) {
      using T = decltype(tag);
      const dim3 grid((unsigned)a.n_idx, (unsigned)((a.dim / 8 + 255) / 256));
      if (a.idx_dtype == kI64)
        return launch_k(gbq8_kernel<T, int64_t>, grid, dim3(256), 0, st, a.data, static_cast<const T*>(a.scales),
                        a.zp, static_cast<const int64_t*>(a.indices), static_cast<T*>(a.out), a.n_idx, a.rows,
                        a.dim, a.block, a.err);
      return launch_k(gbq8_kernel<T, int32_t>, grid, dim3(256), 0, st, a.data, static_cast<const T*>(a.scales),
                      a.zp, static_cast<const int32_t*>(a.indices), static_cast<T*>(a.out), a.n_idx, a.rows, a.dim,
                      a.block, a.err);
    });
  }
  const int blocks = (int)((a.n_idx * 32 + 255) / 256);
  return by_dtype(a.dtype, [&](auto tag) {
    using T = decltype(tag);
    if (a.idx_dtype == kI64)
      return launch_k(gbq_kernel<T, int64_t>, dim3(blocks), dim3(256), 0, st, a.data, static_cast<const T*>(a.scales),
                      a.zp, static_cast<const int64_t*>(a.indices), static_cast<T*>(a.out), a.n_idx, a.rows, a.dim,
                      a.block, a.err);
    return launch_k(gbq_kernel<T, int32_t>, dim3(blocks), dim3(256), 0, st, a.data, static_cast<const T*>(a.scales),
                    a.zp, static_cast<const int32_t*>(a.indices), static_cast<T*>(a.out), a.n_idx, a.rows, a.dim,
                    a.block, a.err);
  });
}

}  // namespace b200ep
