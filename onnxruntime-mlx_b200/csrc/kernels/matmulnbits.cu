// MatMulNBits kernels for sm_100a (com.microsoft MatMulNBits; reference translation
// rust/src/ops/quant.rs:986-1130).
//
//   mnb_gemv_kernel   decode path, M <= 4 (up to 16 rows in chunks of 4): streams the packed weight rows with 128-bit
//                     non-allocating loads (16 B = 32 int4 values per lane per load), dequantises
//                     in registers and reduces with warp shuffles.  HBM-bound.
//   mnb_wide_kernel   many rows (M > 16), int4, K % 32 == 0: SIMT 128 x 128 tiles, 8 x 8 per thread.
//   mnb_tile_kernel   any other M / layout: SIMT tiled GEMM over a shared-memory dequantised weight
//                     tile.  Used for shapes the GEMV does not cover (and as the parity path for
//                     large M until the tensor-core GEMM takes them).
//   mnb_dequant_kernel  W[N,K] = (q - zp) * scale, bit-exact against the CPU oracle.
//
// Weight layout (ONNX Runtime's, unchanged on device): row n holds nblocks blocks of
// block*bits/8 bytes, values packed low-to-high along K (int4: low nibble = even k).
#include <algorithm>

#include "../common.cuh"
#include "kernels.h"

namespace b200ep {

namespace {

template <int BITS>
__device__ __forceinline__ int load_q(const uint8_t* row, int64_t k) {
  if (BITS == 4) {
    uint8_t b = row[k >> 1];
    return (k & 1) ? (b >> 4) : (b & 0x0f);
  }
  return row[k];
}

template <int BITS>
__device__ __forceinline__ int load_zp(const uint8_t* zp, int64_t n, int64_t blk, int64_t nblocks) {
  if (!zp) return 1 << (BITS - 1);
  if (BITS == 4) {
    uint8_t b = zp[n * ((nblocks + 1) >> 1) + (blk >> 1)];
    return (blk & 1) ? (b >> 4) : (b & 0x0f);
  }
  return zp[n * nblocks + blk];
}

// fp32 value 2^23 + byte j of w (j in 0..3) through one byte permute.
__device__ __forceinline__ float magic_byte(uint32_t w, int j) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(w), "r"(0x4B000000u), "r"(0x7440u + j));
  return __uint_as_float(r);
}

}  // namespace

// ---- dequant ------------------------------------------------------------------------------------
template <typename TS, typename TO, int BITS>
__global__ void mnb_dequant_kernel(const uint8_t* __restrict__ B, const TS* __restrict__ scales,
                                   const uint8_t* __restrict__ zp, TO* __restrict__ W, int64_t N,
                                   int64_t K, int block, int64_t nblocks) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = N * K;
  const int64_t rowbytes = nblocks * block * BITS / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t n = i / K, k = i - n * K;
    int64_t blk = k / block;
    int q = load_q<BITS>(B + n * rowbytes, k);
    int z = load_zp<BITS>(zp, n, blk, nblocks);
    float w = (float)(q - z) * to_f<TS>(scales[n * nblocks + blk]);
    if constexpr (sizeof(TO) == 4) W[i] = w; else W[i] = from_f<TO>(w);
  }
}

// ---- decode GEMV ----------------------------------------------------------------------------
// Persistent grid (one wave).  Warp gw owns the row tuples gw, gw + total_warps, ...; a tuple is
// R consecutive weight rows processed together so every activation value read from shared memory
// serves R rows.  A warp walks its (tuple, group) items — a group is U 16-byte chunks per lane
// of each of the R rows, lane-contiguous so one warp load covers 512 contiguous bytes — with the
// next item's weights, scales and zero points already in flight (register double buffer).  The
// first item's loads are issued before the activation is staged, so HBM streaming starts at once.
// The activation is staged once per CTA as fp32 with a 4-float pad per chunk row (conflict-free
// 128-bit reads for the 8 lanes of a shared-memory phase).  Dequant: 2^23 + q built by one byte
// permute, minus (2^23 + zp) in one exact add, then fp32 FMAs; the block scale is applied once
// per block.
constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvU = 2;

template <int BITS, int BLOCK, int R, bool HAS_ZP>
struct GemvBuf {
  static constexpr int VPC = 128 / BITS;
  static constexpr int NBC = BLOCK >= VPC ? 1 : VPC / BLOCK;
  uint4 w[R][kGemvU];
  float s[R][kGemvU][NBC];
  int z[R][kGemvU][NBC];
};

template <typename T, int BITS, int BLOCK, int R, bool HAS_ZP>
__device__ __forceinline__ void gemv_load(GemvBuf<BITS, BLOCK, R, HAS_ZP>& b, const uint8_t* __restrict__ B,
                                          const T* __restrict__ scales, const uint8_t* __restrict__ zp,
                                          int row0, int g, int lane, int N, int cpr, int nblocks) {
  constexpr int VPC = 128 / BITS;
  constexpr int NBC = BLOCK >= VPC ? 1 : VPC / BLOCK;
  const int zcols = (nblocks + 1) >> 1;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = row0 + r;
#pragma unroll
    for (int u = 0; u < kGemvU; ++u) {
      const int c = (g * kGemvU + u) * 32 + lane;
      if (row < N && c < cpr) {
        b.w[r][u] = ld_stream_u4(B + ((size_t)row * cpr + c) * 16);
#pragma unroll
        for (int bc = 0; bc < NBC; ++bc) {
          const int blk = c * VPC / BLOCK + bc;
          b.s[r][u][bc] = to_f<T>(scales[(size_t)row * nblocks + blk]);
          if (HAS_ZP) {
            if (BITS == 4) {
              const uint8_t zb = zp[(size_t)row * zcols + (blk >> 1)];
              b.z[r][u][bc] = (blk & 1) ? (zb >> 4) : (zb & 0x0f);
            } else {
              b.z[r][u][bc] = zp[(size_t)row * nblocks + blk];
            }
          } else {
            b.z[r][u][bc] = 1 << (BITS - 1);
          }
        }
      } else {
        b.w[r][u] = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int bc = 0; bc < NBC; ++bc) {
          b.s[r][u][bc] = 0.f;
          b.z[r][u][bc] = 0;
        }
      }
    }
  }
}

template <int BITS, int BLOCK, int MT, int R, bool HAS_ZP>
__device__ __forceinline__ void gemv_compute(const GemvBuf<BITS, BLOCK, R, HAS_ZP>& b, const float* __restrict__ xs,
                                             int g, int lane, int cpr, float (&acc)[R][MT]) {
  constexpr int VPC = 128 / BITS;
  constexpr int XS = VPC + 4;
  constexpr int NBC = BLOCK >= VPC ? 1 : VPC / BLOCK;
  constexpr int WPB = 4 / NBC;
#pragma unroll
  for (int u = 0; u < kGemvU; ++u) {
    const int c = (g * kGemvU + u) * 32 + lane;
    if (c >= cpr) break;
#pragma unroll
    for (int bc = 0; bc < NBC; ++bc) {
      float part[R][MT];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < MT; ++m) part[r][m] = 0.f;
#pragma unroll
      for (int wi = 0; wi < WPB; ++wi) {
        const int wj = bc * WPB + wi;
        if (BITS == 4) {
          float4 xa[MT], xb[MT];
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            const float4* xp = reinterpret_cast<const float4*>(xs + ((size_t)m * cpr + c) * XS + wj * 8);
            xa[m] = xp[0];
            xb[m] = xp[1];
          }
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const uint32_t w = wj == 0 ? b.w[r][u].x : wj == 1 ? b.w[r][u].y : wj == 2 ? b.w[r][u].z : b.w[r][u].w;
            const float bias = -(8388608.0f + (float)b.z[r][u][bc]);
            const uint32_t lo = w & 0x0f0f0f0fu, hi = (w >> 4) & 0x0f0f0f0fu;
            float d[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              d[2 * j] = magic_byte(lo, j) + bias;
              d[2 * j + 1] = magic_byte(hi, j) + bias;
            }
#pragma unroll
            for (int m = 0; m < MT; ++m) {
              float p = part[r][m];
              p = fmaf(xa[m].x, d[0], p);
              p = fmaf(xa[m].y, d[1], p);
              p = fmaf(xa[m].z, d[2], p);
              p = fmaf(xa[m].w, d[3], p);
              p = fmaf(xb[m].x, d[4], p);
              p = fmaf(xb[m].y, d[5], p);
              p = fmaf(xb[m].z, d[6], p);
              p = fmaf(xb[m].w, d[7], p);
              part[r][m] = p;
            }
          }
        } else {
          float4 xa[MT];
#pragma unroll
          for (int m = 0; m < MT; ++m)
            xa[m] = *reinterpret_cast<const float4*>(xs + ((size_t)m * cpr + c) * XS + wj * 4);
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const uint32_t w = wj == 0 ? b.w[r][u].x : wj == 1 ? b.w[r][u].y : wj == 2 ? b.w[r][u].z : b.w[r][u].w;
            const float bias = -(8388608.0f + (float)b.z[r][u][bc]);
            float d[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) d[j] = magic_byte(w, j) + bias;
#pragma unroll
            for (int m = 0; m < MT; ++m) {
              float p = part[r][m];
              p = fmaf(xa[m].x, d[0], p);
              p = fmaf(xa[m].y, d[1], p);
              p = fmaf(xa[m].z, d[2], p);
              p = fmaf(xa[m].w, d[3], p);
              part[r][m] = p;
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[r][m] = fmaf(part[r][m], b.s[r][u][bc], acc[r][m]);
    }
  }
}

template <typename T, int BITS, int BLOCK, int MT, int R, bool HAS_ZP>
__global__ void __launch_bounds__(kGemvThreads, 2)
mnb_gemv_kernel(const T* __restrict__ A, const uint8_t* __restrict__ B,
                const T* __restrict__ scales, const uint8_t* __restrict__ zp,
                T* __restrict__ Y, int M, int N, int K, int nblocks, int cpr) {
  pdl_wait();
  pdl_trigger();
  constexpr int VPC = 128 / BITS;
  constexpr int XS = VPC + 4;
  extern __shared__ __align__(16) float xs[];  // [MT][cpr][XS]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kGemvWarps + warp;
  const int tw = gridDim.x * kGemvWarps;
  const int ntuples = (N + R - 1) / R;
  const int gpr = (cpr + 32 * kGemvU - 1) / (32 * kGemvU);
  const int my_tuples = gw < ntuples ? (ntuples - 1 - gw) / tw + 1 : 0;
  const int nitems = my_tuples * gpr;

  using Buf = GemvBuf<BITS, BLOCK, R, HAS_ZP>;
  Buf b0, b1;
  if (nitems > 0) gemv_load<T>(b0, B, scales, zp, gw * R, 0, lane, N, cpr, nblocks);

  // stage the activation rows (fp32, padded) while the first weights are in flight
  for (int m = 0; m < MT; ++m) {
    for (int k = threadIdx.x; k < cpr * VPC; k += kGemvThreads) {
      const int c = k / VPC, j = k - c * VPC;
      xs[((size_t)m * cpr + c) * XS + j] = (m < M && k < K) ? to_f<T>(A[(size_t)m * K + k]) : 0.f;
    }
  }
  __syncthreads();

  float acc[R][MT];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[r][m] = 0.f;

  auto finish_item = [&](int item) {
    const int g = item % gpr;
    if (g != gpr - 1) return;
    const int row0 = (gw + (item / gpr) * tw) * R;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const float v = warp_sum(acc[r][m]);
        acc[r][m] = 0.f;
        if (lane == 0 && m < M && row0 + r < N) Y[(size_t)m * N + row0 + r] = from_f<T>(v);
      }
  };

  for (int item = 0; item < nitems; item += 2) {
    // item -> buffer b0, item+1 -> buffer b1 (loaded one step ahead)
    if (item + 1 < nitems) {
      const int it = item + 1;
      gemv_load<T>(b1, B, scales, zp, (gw + (it / gpr) * tw) * R, it % gpr, lane, N, cpr, nblocks);
    }
    gemv_compute<BITS, BLOCK, MT, R, HAS_ZP>(b0, xs, item % gpr, lane, cpr, acc);
    finish_item(item);
    if (item + 1 >= nitems) break;
    if (item + 2 < nitems) {
      const int it = item + 2;
      gemv_load<T>(b0, B, scales, zp, (gw + (it / gpr) * tw) * R, it % gpr, lane, N, cpr, nblocks);
    }
    gemv_compute<BITS, BLOCK, MT, R, HAS_ZP>(b1, xs, (item + 1) % gpr, lane, cpr, acc);
    finish_item(item + 1);
  }
}

// ---- generic tiled kernel -------------------------------------------------------------------
// CTA tile 64(m) x 64(n), K step 32; 256 threads each own a 4x4 output micro-tile.
constexpr int kTM = 64, kTN = 64, kTK = 32;

template <typename T, int BITS>
__global__ void __launch_bounds__(256)
mnb_tile_kernel(const T* __restrict__ A, const uint8_t* __restrict__ B,
                const T* __restrict__ scales, const uint8_t* __restrict__ zp,
                T* __restrict__ Y, int M, int N, int K, int block, int nblocks) {
  __shared__ float as[kTK][kTM + 4];
  pdl_wait();
  pdl_trigger();
  __shared__ float ws[kTK][kTN + 4];
  const int m0 = blockIdx.y * kTM, n0 = blockIdx.x * kTN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t rowbytes = (int64_t)nblocks * block * BITS / 8;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += kTK) {
    for (int i = threadIdx.x; i < kTM * kTK; i += 256) {
      int mm = i / kTK, kk = i % kTK;
      int m = m0 + mm, k = k0 + kk;
      as[kk][mm] = (m < M && k < K) ? to_f<T>(A[(size_t)m * K + k]) : 0.f;
    }
    for (int i = threadIdx.x; i < kTN * kTK; i += 256) {
      int nn = i / kTK, kk = i % kTK;
      int n = n0 + nn, k = k0 + kk;
      float w = 0.f;
      if (n < N && k < K) {
        int64_t blk = k / block;
        int q = load_q<BITS>(B + (size_t)n * rowbytes, k);
        int z = load_zp<BITS>(zp, n, blk, nblocks);
        w = (float)(q - z) * to_f<T>(scales[(size_t)n * nblocks + blk]);
      }
      ws[kk][nn] = w;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kTK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = as[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = ws[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int n = n0 + tx * 4 + j;
      if (n < N) Y[(size_t)m * N + n] = from_f<T>(acc[i][j]);
    }
  }
}

// ---- wide tiled kernel (many rows) ----------------------------------------------------------
// CTA tile 128(m) x 128(n), K step 32, 256 threads each owning an 8 x 8 output micro-tile: 64 FMAs
// per four 16-byte shared-memory loads.  Weight tile: thread t dequantises row n0 + t / 2, k half
// t % 2 (16 values: one 8-byte load, one scale, one zero point; blocks of 16 or more keep a half
// inside one block); activation tile: two rows of 8 values per thread.  The next K step's global
// loads are issued before the current step's FMAs.  Requires K % 32 == 0, block % 16 == 0, A 16-byte
// aligned rows (K % 4 == 0), 4-bit weights.
constexpr int kWM = 128, kWN = 128, kWK = 32;

template <typename T>
__global__ void __launch_bounds__(256)
mnb_wide_kernel(const T* __restrict__ A, const uint8_t* __restrict__ B, const T* __restrict__ scales,
                const uint8_t* __restrict__ zp, T* __restrict__ Y, int M, int N, int K, int block, int nblocks) {
  __shared__ __align__(16) float as[kWK][kWM + 4];
  __shared__ __align__(16) float ws[kWK][kWN + 4];
  pdl_wait();
  pdl_trigger();
  const int m0 = blockIdx.y * kWM, n0 = blockIdx.x * kWN;
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const int64_t rowbytes = (int64_t)nblocks * block / 2;
  // weight loader: row wn, k half wh
  const int wn = tid >> 1, wh = tid & 1;
  const int n = n0 + wn;
  // activation loader: rows am + 64 i (i < 2), k chunk ak (8 floats)
  const int am = tid >> 2, ak = (tid & 3) * 8;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  uint2 wq = make_uint2(0, 0);
  float wsc = 0.f;
  int wz = 8;
  float av[2][8];
  auto load = [&](int k0) {
    if (n < N) {
      const int k = k0 + wh * 16;
      const int64_t blk = k / block;
      wq = *reinterpret_cast<const uint2*>(B + (size_t)n * rowbytes + k / 2);
      wsc = to_f<T>(scales[(size_t)n * nblocks + blk]);
      wz = zp ? ((blk & 1) ? zp[(size_t)n * ((nblocks + 1) >> 1) + (blk >> 1)] >> 4
                           : zp[(size_t)n * ((nblocks + 1) >> 1) + (blk >> 1)] & 15)
              : 8;
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int m = m0 + am + 64 * i;
#pragma unroll
      for (int j = 0; j < 8; ++j) av[i][j] = 0.f;
      if (m < M) {
        const T* src = A + (size_t)m * K + k0 + ak;
#pragma unroll
        for (int j = 0; j < 8; ++j) av[i][j] = to_f<T>(src[j]);
      }
    }
  };
  load(0);
  for (int k0 = 0; k0 < K; k0 += kWK) {
    // publish this step's tiles
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t word = j < 8 ? wq.x : wq.y;
      const int q = (word >> (4 * (j & 7))) & 15;
      ws[wh * 16 + j][wn] = n < N ? (float)(q - wz) * wsc : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) as[ak + j][am + 64 * i] = av[i][j];
    __syncthreads();
    if (k0 + kWK < K) load(k0 + kWK);
#pragma unroll 4
    for (int kk = 0; kk < kWK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&as[kk][ty * 8]);
      const float4 a1 = *reinterpret_cast<const float4*>(&as[kk][ty * 8 + 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&ws[kk][tx * 8]);
      const float4 b1 = *reinterpret_cast<const float4*>(&ws[kk][tx * 8 + 4]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + ty * 8 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int nn = n0 + tx * 8 + j;
      if (nn < N) Y[(size_t)m * N + nn] = from_f<T>(acc[i][j]);
    }
  }
}

// ---- host launchers -------------------------------------------------------------------------
namespace {


template <typename T, int BITS, int BLOCK, int MT, bool HAS_ZP>
cudaError_t launch_gemv_t(const MnbArgs& a, cudaStream_t st) {
  constexpr int VPC = 128 / BITS;
  constexpr int XS = VPC + 4;
  constexpr int R = MT <= 2 ? 2 : 1;
  const int64_t nblocks = (a.K + BLOCK - 1) / BLOCK;
  const int cpr = (int)(nblocks * BLOCK * BITS / 8 / 16);
  const size_t smem = (size_t)MT * cpr * XS * sizeof(float);
  auto kern = mnb_gemv_kernel<T, BITS, BLOCK, MT, R, HAS_ZP>;
  static int configured_smem = 0;  // per instantiation
  if ((int)smem > configured_smem && smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured_smem = (int)smem;
  }
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGemvThreads, smem);
  if (e != cudaSuccess) return e;
  per_sm = std::max(1, per_sm);
  const int64_t ntuples = (a.N + R - 1) / R;
  const int64_t want = (ntuples + kGemvWarps - 1) / kGemvWarps;
  const int grid = (int)std::min<int64_t>(want, (int64_t)per_sm * num_sms());
  return launch_k(kern, dim3(grid), dim3(kGemvThreads), smem, st, static_cast<const T*>(a.A), a.B,
                  static_cast<const T*>(a.scales), a.zp, static_cast<T*>(a.Y), (int)a.M, (int)a.N, (int)a.K,
                  (int)nblocks, cpr);
}

template <typename T, int BITS, int BLOCK, bool HAS_ZP>
cudaError_t launch_gemv_m(const MnbArgs& a, cudaStream_t st) {
  if (a.M <= 1) return launch_gemv_t<T, BITS, BLOCK, 1, HAS_ZP>(a, st);
  if (a.M <= 2) return launch_gemv_t<T, BITS, BLOCK, 2, HAS_ZP>(a, st);
  return launch_gemv_t<T, BITS, BLOCK, 4, HAS_ZP>(a, st);
}

template <typename T, int BITS, int BLOCK>
cudaError_t launch_gemv_z(const MnbArgs& a, cudaStream_t st) {
  return a.zp ? launch_gemv_m<T, BITS, BLOCK, true>(a, st) : launch_gemv_m<T, BITS, BLOCK, false>(a, st);
}

template <typename T, int BITS>
cudaError_t launch_gemv_b(const MnbArgs& a, cudaStream_t st) {
  switch (a.block) {
    case 16: return launch_gemv_z<T, BITS, 16>(a, st);
    case 32: return launch_gemv_z<T, BITS, 32>(a, st);
    case 64: return launch_gemv_z<T, BITS, 64>(a, st);
    case 128: return launch_gemv_z<T, BITS, 128>(a, st);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
cudaError_t launch_dtype(const MnbArgs& a, cudaStream_t st) {
  const int64_t nblocks = (a.K + a.block - 1) / a.block;
  const int64_t rowbytes = nblocks * a.block * a.bits / 8;
  const int64_t mt = a.M <= 1 ? 1 : a.M <= 2 ? 2 : 4;
  const int64_t stage_bytes = mt * (rowbytes / 16) * (128 / a.bits + 4) * 4;
  const bool gemv_ok = rowbytes % 16 == 0 && stage_bytes <= 200 * 1024 && (reinterpret_cast<uintptr_t>(a.B) % 16) == 0;
  if (gemv_ok && a.M <= 4) return a.bits == 4 ? launch_gemv_b<T, 4>(a, st) : launch_gemv_b<T, 8>(a, st);
  if (gemv_ok && a.M <= 16) {
    // up to 16 rows: the GEMV over chunks of 4 activation rows (the weights, at most a few tens of
    // MB for decode shapes, come from L2 after the first chunk)
    for (int64_t m0 = 0; m0 < a.M; m0 += 4) {
      MnbArgs c = a;
      c.A = static_cast<const T*>(a.A) + m0 * a.K;
      c.Y = static_cast<T*>(a.Y) + m0 * a.N;
      c.M = std::min<int64_t>(4, a.M - m0);
      cudaError_t e = a.bits == 4 ? launch_gemv_b<T, 4>(c, st) : launch_gemv_b<T, 8>(c, st);
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
  if (a.bits == 4 && a.K % kWK == 0 && a.block % 16 == 0 && a.K % a.block == 0 && a.M > 16) {
    dim3 wgrid((unsigned)div_up(a.N, kWN), (unsigned)div_up(a.M, kWM));
    return launch_k(mnb_wide_kernel<T>, wgrid, dim3(256), 0, st, static_cast<const T*>(a.A), a.B,
                    static_cast<const T*>(a.scales), a.zp, static_cast<T*>(a.Y), (int)a.M, (int)a.N, (int)a.K,
                    a.block, (int)nblocks);
  }
  dim3 grid((unsigned)div_up(a.N, kTN), (unsigned)div_up(a.M, kTM));
  auto kern = a.bits == 4 ? mnb_tile_kernel<T, 4> : mnb_tile_kernel<T, 8>;
  return launch_k(kern, grid, dim3(256), 0, st, static_cast<const T*>(a.A), a.B, static_cast<const T*>(a.scales),
                  a.zp, static_cast<T*>(a.Y), (int)a.M, (int)a.N, (int)a.K, a.block, (int)nblocks);
}

template <typename TS, typename TO>
cudaError_t launch_dequant_t(const MnbDequantArgs& a, cudaStream_t st) {
  const int64_t nblocks = (a.K + a.block - 1) / a.block;
  const int64_t total = a.N * a.K;
  int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  auto kern = a.bits == 4 ? mnb_dequant_kernel<TS, TO, 4> : mnb_dequant_kernel<TS, TO, 8>;
  return launch_k(kern, dim3(grid), dim3(256), 0, st, a.B, static_cast<const TS*>(a.scales), a.zp,
                  static_cast<TO*>(a.W), a.N, a.K, a.block, nblocks);
}

template <typename TS>
cudaError_t launch_dequant_s(const MnbDequantArgs& a, cudaStream_t st) {
  switch (a.out_dtype) {
    case kF32: return launch_dequant_t<TS, float>(a, st);
    case kF16: return launch_dequant_t<TS, __half>(a, st);
    case kBF16: return launch_dequant_t<TS, __nv_bfloat16>(a, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_matmulnbits(const MnbArgs& a, cudaStream_t st) {
  if (a.M == 0) return cudaSuccess;
  switch (a.dtype) {
    case kF32: return launch_dtype<float>(a, st);
    case kF16: return launch_dtype<__half>(a, st);
    case kBF16: return launch_dtype<__nv_bfloat16>(a, st);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_matmulnbits_dequant(const MnbDequantArgs& a, cudaStream_t st) {
  switch (a.scale_dtype) {
    case kF32: return launch_dequant_s<float>(a, st);
    case kF16: return launch_dequant_s<__half>(a, st);
    case kBF16: return launch_dequant_s<__nv_bfloat16>(a, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace b200ep
