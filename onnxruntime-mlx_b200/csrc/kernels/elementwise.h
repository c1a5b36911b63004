// Launchers for the elementwise glue kernels used by the EP plan executor.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200ep {

struct DeviceErrorSlot;

enum BinaryOp { kOpAdd = 0, kOpSub = 1, kOpMul = 2 };

// Output dims and per-input element strides (0 on broadcast dims), rank <= 6, row-major.
struct BinaryGeom {
  int rank = 0;
  int64_t total = 0;
  int64_t out_dims[6] = {};
  int64_t a_strides[6] = {};
  int64_t b_strides[6] = {};
};

cudaError_t launch_binary(const void* a, const void* b, void* y, int dtype, const BinaryGeom& g, int op,
                          cudaStream_t st);
cudaError_t launch_sigmoid(const void* x, void* y, int dtype, int64_t n, cudaStream_t st);
cudaError_t launch_silu_mul(const void* gu, void* h, int dtype, int64_t rows, int64_t n, cudaStream_t st);
cudaError_t launch_cast(const void* x, int in_dt, void* y, int out_dt, int64_t n, cudaStream_t st);
// SiLU(gate) * up over gate / up columns interleaved in groups of 8 ([rows, 2n] -> [rows, n])
cudaError_t launch_silu_mul_interleaved(const void* gu, void* h, int dtype, int64_t rows, int64_t n,
                                        cudaStream_t st);

// Integer glue (index_ops.cu): exact int32 / int64 arithmetic for the attention-mask and
// shape-vector chains of exported decoders.
struct IdxList {
  int n = 0;
  int64_t v[8] = {};
};
cudaError_t launch_binary_int(const void* a, const void* b, void* y, int dtype, const BinaryGeom& g, int op,
                              cudaStream_t st);
cudaError_t launch_cast_int(const void* x, int in_dt, void* y, int out_dt, int64_t n, cudaStream_t st);
// y[r] = sum of row r of x ([rows, len] row-major); len is read from *len_dev when it is non-null
cudaError_t launch_reduce_sum_rows(const void* x, int x_dt, void* y, int y_dt, int64_t rows, int64_t len,
                                   const int64_t* len_dev, cudaStream_t st);
cudaError_t launch_gather_idx(const void* x, void* y, int dtype, const IdxList& idx, cudaStream_t st);
cudaError_t launch_copy_bytes(const void* x, void* y, int64_t bytes, cudaStream_t st);

struct GbqArgs {
  const uint8_t* data;
  const void* scales;
  const uint8_t* zp;
  const void* indices;
  int idx_dtype;
  void* out;
  int dtype;
  int64_t n_idx, rows, dim;
  int block;
  DeviceErrorSlot* err;
};
cudaError_t launch_gather_block_quantized(const GbqArgs& a, cudaStream_t st);

}  // namespace b200ep
