// MatMulNBits kernels for sm_100a (com.microsoft MatMulNBits; reference translation
// rust/src/ops/quant.rs:986-1130).
//
//   mnb_gemv_kernel   decode path, M <= 4: streams the packed weight rows with 128-bit
//                     non-allocating loads (16 B = 32 int4 values per lane per load), dequantises
//                     in registers and reduces with warp shuffles.  HBM-bound.
//   mnb_tile_kernel   any M / layout: SIMT tiled GEMM over a shared-memory dequantised weight
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
// Grid: one CTA per group of (8 / WPR) weight rows; WPR warps cooperate on one row (split along
// K) so small-N projections still fill the GPU.  The activation rows are staged in shared
// memory as fp32 in segments of SEGC 16-byte chunks; the smem row for each chunk is padded by
// 4 floats so that the 128-bit reads of 8 consecutive lanes hit distinct banks.
constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;

template <typename T, int BITS, int BLOCK, int MT, bool HAS_ZP>
__global__ void __launch_bounds__(kGemvThreads, 3)
mnb_gemv_kernel(const T* __restrict__ A, const uint8_t* __restrict__ B,
                const T* __restrict__ scales, const uint8_t* __restrict__ zp,
                T* __restrict__ Y, int M, int N, int K, int nblocks, int chunks_per_row,
                int segc, int wpr) {
  constexpr int VPC = 128 / BITS;        // values per 16-byte chunk
  constexpr int XS = VPC + 4;            // padded floats per chunk in smem
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;                      // [MT][segc][XS]
  float* red = smem + MT * segc * XS;    // [kGemvWarps][MT] cross-warp partials

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows_per_cta = kGemvWarps / wpr;
  const int n = blockIdx.x * rows_per_cta + warp / wpr;
  const int sub = warp % wpr;
  const bool row_ok = n < N;
  const size_t rowbytes = (size_t)chunks_per_row * 16;
  const uint8_t* brow = B + (size_t)(row_ok ? n : 0) * rowbytes;
  const int zcols = (nblocks + 1) >> 1;

  float acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = 0.f;

  for (int seg0 = 0; seg0 < chunks_per_row; seg0 += segc) {
    const int nseg = min(segc, chunks_per_row - seg0);
    __syncthreads();
    // stage A[:, seg] as fp32 (zero beyond K and beyond M)
    for (int i = threadIdx.x; i < MT * nseg * VPC; i += kGemvThreads) {
      int m = i / (nseg * VPC);
      int r = i - m * nseg * VPC;
      int c = r / VPC, j = r - c * VPC;
      int k = (seg0 + c) * VPC + j;
      float v = (m < M && k < K) ? to_f<T>(A[(size_t)m * K + k]) : 0.f;
      xs[(m * segc + c) * XS + j] = v;
    }
    __syncthreads();
    if (!row_ok) continue;

    constexpr int U = 4;
    for (int c0 = sub * 32 + lane; c0 < nseg; c0 += 32 * wpr * U) {
      uint4 wv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        int c = c0 + u * 32 * wpr;
        if (c < nseg) wv[u] = ld_stream_u4(brow + (size_t)(seg0 + c) * 16);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        int c = c0 + u * 32 * wpr;
        if (c >= nseg) break;
        const int cg = seg0 + c;                 // global chunk index
        const int k0 = cg * VPC;
        const uint32_t words[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
        // blocks covered by this chunk: one (BLOCK >= VPC) or VPC/BLOCK (block 16, int4)
        constexpr int NBC = BLOCK >= VPC ? 1 : VPC / BLOCK;
        constexpr int WPB = 4 / NBC;             // 32-bit words per block inside the chunk
#pragma unroll
        for (int bc = 0; bc < NBC; ++bc) {
          const int blk = k0 / BLOCK + bc;
          const float s = to_f<T>(scales[(size_t)n * nblocks + blk]);
          int z;
          if (HAS_ZP) {
            if (BITS == 4) {
              uint8_t zb = zp[(size_t)n * zcols + (blk >> 1)];
              z = (blk & 1) ? (zb >> 4) : (zb & 0x0f);
            } else {
              z = zp[(size_t)n * nblocks + blk];
            }
          } else {
            z = 1 << (BITS - 1);
          }
          const float bias = -(8388608.0f + (float)z);
          float part[MT];
#pragma unroll
          for (int m = 0; m < MT; ++m) part[m] = 0.f;
#pragma unroll
          for (int wi = 0; wi < WPB; ++wi) {
            const int wj = bc * WPB + wi;
            const uint32_t w = words[wj];
            if (BITS == 4) {
              const uint32_t lo = w & 0x0f0f0f0fu;         // nibbles k = 0,2,4,6 of the word
              const uint32_t hi = (w >> 4) & 0x0f0f0f0fu;  // nibbles k = 1,3,5,7
              float d[8];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                d[2 * j] = magic_byte(lo, j) + bias;
                d[2 * j + 1] = magic_byte(hi, j) + bias;
              }
#pragma unroll
              for (int m = 0; m < MT; ++m) {
                const float4* xp = reinterpret_cast<const float4*>(xs + (m * segc + c) * XS + wj * 8);
                float4 xa = xp[0], xb = xp[1];
                part[m] = fmaf(xa.x, d[0], part[m]);
                part[m] = fmaf(xa.y, d[1], part[m]);
                part[m] = fmaf(xa.z, d[2], part[m]);
                part[m] = fmaf(xa.w, d[3], part[m]);
                part[m] = fmaf(xb.x, d[4], part[m]);
                part[m] = fmaf(xb.y, d[5], part[m]);
                part[m] = fmaf(xb.z, d[6], part[m]);
                part[m] = fmaf(xb.w, d[7], part[m]);
              }
            } else {
              float d[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) d[j] = magic_byte(w, j) + bias;
#pragma unroll
              for (int m = 0; m < MT; ++m) {
                float4 xa = *reinterpret_cast<const float4*>(xs + (m * segc + c) * XS + wj * 4);
                part[m] = fmaf(xa.x, d[0], part[m]);
                part[m] = fmaf(xa.y, d[1], part[m]);
                part[m] = fmaf(xa.z, d[2], part[m]);
                part[m] = fmaf(xa.w, d[3], part[m]);
              }
            }
          }
#pragma unroll
          for (int m = 0; m < MT; ++m) acc[m] = fmaf(part[m], s, acc[m]);
        }
      }
    }
  }

#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = warp_sum(acc[m]);
  if (wpr == 1) {
    if (row_ok && lane == 0) {
#pragma unroll
      for (int m = 0; m < MT; ++m)
        if (m < M) Y[(size_t)m * N + n] = from_f<T>(acc[m]);
    }
    return;
  }
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < MT; ++m) red[warp * MT + m] = acc[m];
  }
  __syncthreads();
  if (row_ok && sub == 0 && lane < MT && lane < M) {
    float v = 0.f;
    for (int s2 = 0; s2 < wpr; ++s2) v += red[(warp + s2) * MT + lane];
    Y[(size_t)lane * N + n] = from_f<T>(v);
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

// ---- host launchers -------------------------------------------------------------------------
namespace {

template <typename T, int BITS, int BLOCK, int MT, bool HAS_ZP>
cudaError_t launch_gemv_t(const MnbArgs& a, cudaStream_t st) {
  constexpr int VPC = 128 / BITS;
  constexpr int XS = VPC + 4;
  const int64_t nblocks = (a.K + BLOCK - 1) / BLOCK;
  const int chunks_per_row = (int)(nblocks * BLOCK * BITS / 8 / 16);
  // segment size: keep the fp32 activation stage near 40 KB, whole 32-chunk multiples
  int segc = (40 * 1024) / (MT * XS * 4);
  segc = std::max(32, (segc / 32) * 32);
  segc = std::min(segc, ((chunks_per_row + 31) / 32) * 32);
  // warps per row: enough warps in flight for small N
  int wpr = 1;
  while (wpr < 8 && (int64_t)a.N * wpr < 148 * 48 && chunks_per_row >= 64 * wpr) wpr *= 2;
  const int rows_per_cta = kGemvWarps / wpr;
  const size_t smem = (size_t)(MT * segc * XS + kGemvWarps * MT) * sizeof(float);
  auto kern = mnb_gemv_kernel<T, BITS, BLOCK, MT, HAS_ZP>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  dim3 grid((unsigned)div_up(a.N, rows_per_cta));
  kern<<<grid, kGemvThreads, smem, st>>>(
      static_cast<const T*>(a.A), a.B, static_cast<const T*>(a.scales), a.zp,
      static_cast<T*>(a.Y), (int)a.M, (int)a.N, (int)a.K, (int)nblocks, chunks_per_row, segc, wpr);
  return cudaGetLastError();
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
  const bool gemv_ok = a.M <= 4 && rowbytes % 16 == 0 && a.K <= (1 << 24) &&
                       (reinterpret_cast<uintptr_t>(a.B) % 16) == 0;
  if (gemv_ok) return a.bits == 4 ? launch_gemv_b<T, 4>(a, st) : launch_gemv_b<T, 8>(a, st);
  dim3 grid((unsigned)div_up(a.N, kTN), (unsigned)div_up(a.M, kTM));
  if (a.bits == 4)
    mnb_tile_kernel<T, 4><<<grid, 256, 0, st>>>(
        static_cast<const T*>(a.A), a.B, static_cast<const T*>(a.scales), a.zp,
        static_cast<T*>(a.Y), (int)a.M, (int)a.N, (int)a.K, a.block, (int)nblocks);
  else
    mnb_tile_kernel<T, 8><<<grid, 256, 0, st>>>(
        static_cast<const T*>(a.A), a.B, static_cast<const T*>(a.scales), a.zp,
        static_cast<T*>(a.Y), (int)a.M, (int)a.N, (int)a.K, a.block, (int)nblocks);
  return cudaGetLastError();
}

template <typename TS, typename TO>
cudaError_t launch_dequant_t(const MnbDequantArgs& a, cudaStream_t st) {
  const int64_t nblocks = (a.K + a.block - 1) / a.block;
  const int64_t total = a.N * a.K;
  int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  if (a.bits == 4)
    mnb_dequant_kernel<TS, TO, 4><<<grid, 256, 0, st>>>(a.B, static_cast<const TS*>(a.scales), a.zp,
                                                        static_cast<TO*>(a.W), a.N, a.K, a.block, nblocks);
  else
    mnb_dequant_kernel<TS, TO, 8><<<grid, 256, 0, st>>>(a.B, static_cast<const TS*>(a.scales), a.zp,
                                                        static_cast<TO*>(a.W), a.N, a.K, a.block, nblocks);
  return cudaGetLastError();
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
