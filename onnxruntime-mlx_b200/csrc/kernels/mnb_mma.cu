// MatMulNBits on the tensor cores for fp16 / bf16 activations and int4 weights
// (reference: matmulnbits_op, rust/src/ops/quant.rs:986-1130).
//
// Prepacked layout.  The weight is repacked once (the EP does it when it uploads initializers;
// the reference repacks to MLX words at the same point, quant.rs:634-710) into "group records":
// one record per 16-row tile and 64 k (4 k-steps of mma.sync.m16n8k16), tile-major, so that the
// records of a tile — and of a run of consecutive tiles — are contiguous in HBM:
//   bytes [0, 512)    32 lanes x uint4: lane l = 4g + c holds, for each of the 4 k-steps s, the
//                     32-bit word with the 8 nibbles of its A fragment
//                       bits  0- 3: W[16t+g  ][16s+2c  ]   bits 16-19: W[16t+g  ][16s+2c+1]
//                       bits  4- 7: W[16t+g+8][16s+2c  ]   bits 20-23: W[16t+g+8][16s+2c+1]
//                       bits  8-11: W[16t+g  ][16s+2c+8]   bits 24-27: W[16t+g  ][16s+2c+9]
//                       bits 12-15: W[16t+g+8][16s+2c+8]   bits 28-31: W[16t+g+8][16s+2c+9]
//   then, per quantisation block the record covers (slot) and row pair g: the scales of rows g
//   and g+8 as one half2 / bf162, then their zero points as one byte (g + 8 in the high nibble);
//   padded to 16 bytes.  Block 32: 512 + 80 = 592 bytes per 512 weight bytes, the same overhead
//   as ONNX Runtime's scales + packed zero points.
//
// Kernel.  One CTA streams a contiguous run of tiles.  A producer warp copies G records per
// stage with one 1-D bulk copy (cp.async.bulk, the TMA engine) into a ring of shared-memory
// stages guarded by mbarriers (all waits bounded); the bytes in flight live in shared memory, not
// registers.  Four consumer warps take the records of a stage round-robin; per record a lane reads
// its 16-byte A words and the block parameters from shared memory, dequantises with
// (w & 0x000F000F) | magic (two fp16 1024 + q, or 64 + q for the nibbles at bits 4-7) and an exact
// half2 subtract of (magic + zp), runs one MMA per k-step against activation fragments read from
// the (L1-resident) activation rows, and scales the fp32 block accumulator once per block.  At a
// tile's last stage the consumers merge their partial sums in shared memory.
#include <algorithm>

#include "../common.cuh"
#include "kernels.h"
#include "mnb_mma.h"

namespace b200ep {

template <int BLOCK>
struct Rec {
  static constexpr int kSlots = BLOCK >= 64 ? 1 : 64 / BLOCK;  // blocks per record
  static constexpr int kSOff = 512;                            // uint32 scales[slot][8]
  static constexpr int kZOff = 512 + kSlots * 32;              // uint8  zps[slot][8]
  static constexpr int kBytes = 512 + ((kSlots * 40 + 15) / 16) * 16;
  static constexpr int kUnit = BLOCK > 64 ? BLOCK / 64 : 1;   // records per block (kept by one warp)
};

int mnb_record_bytes(int block) {
  switch (block) {
    case 16: return Rec<16>::kBytes;
    case 32: return Rec<32>::kBytes;
    case 64: return Rec<64>::kBytes;
    case 128: return Rec<128>::kBytes;
  }
  return 0;
}

// ---- prepack ----------------------------------------------------------------------------------
template <typename TS, int BLOCK>
__global__ void mnb_prepack_kernel(const uint8_t* __restrict__ B, const TS* __restrict__ scales,
                                   const uint8_t* __restrict__ zp, MnbPacked p) {
  using RC = Rec<BLOCK>;
  constexpr int SPB = BLOCK / 16;
  const int64_t nrec = (int64_t)p.ntiles * p.ksteps4;
  const int64_t rowbytes = (int64_t)p.nblocks_src * BLOCK / 2;
  uint8_t* out = static_cast<uint8_t*>(p.w);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // weight words: 128 per record
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nrec * 128; i += stride) {
    const int64_t rec = i >> 7;
    const int w = (int)(i & 127);
    const int lane = w >> 2, j = w & 3;
    const int64_t t = rec / p.ksteps4;
    const int gi = (int)(rec % p.ksteps4);
    const int s = gi * 4 + j;
    const int g = lane >> 2, c = lane & 3;
    const int64_t r0 = t * 16 + g, r1 = r0 + 8;
    const int k0 = s * 16 + 2 * c;
    auto q = [&](int64_t r, int k) -> uint32_t {
      if (r >= p.N || k >= p.nblocks_src * BLOCK) return 0u;
      const uint8_t b = B[r * rowbytes + (k >> 1)];
      return (k & 1) ? (b >> 4) : (b & 0x0f);
    };
    const uint32_t word = q(r0, k0) | (q(r1, k0) << 4) | (q(r0, k0 + 8) << 8) | (q(r1, k0 + 8) << 12) |
                          (q(r0, k0 + 1) << 16) | (q(r1, k0 + 1) << 20) | (q(r0, k0 + 9) << 24) |
                          (q(r1, k0 + 9) << 28);
    *reinterpret_cast<uint32_t*>(out + rec * RC::kBytes + lane * 16 + j * 4) = word;
  }
  // parameters (and the zero padding) per record
  constexpr int kTail = RC::kBytes - 512;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nrec * kTail; i += stride) {
    const int64_t rec = i / kTail;
    const int off = (int)(i % kTail) + 512;
    const int64_t t = rec / p.ksteps4;
    const int gi = (int)(rec % p.ksteps4);
    uint8_t* dst = out + rec * RC::kBytes + off;
    if (off >= RC::kZOff + RC::kSlots * 8) {
      *dst = 0;
      continue;
    }
    const bool is_z = off >= RC::kZOff;
    if (!is_z && ((off - RC::kSOff) & 3)) continue;  // one thread writes each 4-byte scale word
    const int idx = is_z ? off - RC::kZOff : (off - RC::kSOff) / 4;
    const int slot = idx / 8, g = idx % 8;
    const int blk = SPB <= 4 ? (gi * 4) / SPB + slot : gi / (SPB / 4);
    const int64_t r0 = t * 16 + g, r1 = r0 + 8;
    if (is_z) {
      auto zz = [&](int64_t r) -> uint32_t {
        if (r >= p.N || blk >= p.nblocks_src || !zp) return 8u;
        const uint8_t b = zp[r * ((p.nblocks_src + 1) / 2) + (blk >> 1)];
        return (blk & 1) ? (b >> 4) : (b & 0x0f);
      };
      *dst = (uint8_t)(zz(r0) | (zz(r1) << 4));
    } else {
      auto sc = [&](int64_t r) -> TS {
        if (r >= p.N || blk >= p.nblocks_src) return from_f<TS>(0.f);
        return scales[r * p.nblocks_src + blk];
      };
      TS s0 = sc(r0), s1 = sc(r1);
      uint16_t u0, u1;
      memcpy(&u0, &s0, 2);
      memcpy(&u1, &s1, 2);
      *reinterpret_cast<uint32_t*>(dst) = (uint32_t)u0 | ((uint32_t)u1 << 16);
    }
  }
}

// ---- fragment dequant -------------------------------------------------------------------------
template <typename T> struct Dq;
template <> struct Dq<__half> {
  static __device__ __forceinline__ void run(uint32_t w, uint32_t bias_lo, uint32_t bias_hi, uint32_t (&a)[4]) {
    const uint32_t w8 = w >> 8;
    const uint32_t t0 = (w & 0x000F000Fu) | 0x64006400u;   // 1024 + q   rows g,   k 2c / 2c+1
    const uint32_t t1 = (w & 0x00F000F0u) | 0x54005400u;   //   64 + q   rows g+8, k 2c / 2c+1
    const uint32_t t2 = (w8 & 0x000F000Fu) | 0x64006400u;  // 1024 + q   rows g,   k 2c+8 / 2c+9
    const uint32_t t3 = (w8 & 0x00F000F0u) | 0x54005400u;  //   64 + q   rows g+8, k 2c+8 / 2c+9
    asm("sub.f16x2 %0, %1, %2;" : "=r"(a[0]) : "r"(t0), "r"(bias_lo));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(a[1]) : "r"(t1), "r"(bias_hi));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(a[2]) : "r"(t2), "r"(bias_lo));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(a[3]) : "r"(t3), "r"(bias_hi));
  }
  // bias_lo = (1024 + z_g) in both halves, bias_hi = (64 + z_{g+8}) in both halves
  static __device__ __forceinline__ void bias(uint32_t zb, uint32_t& lo, uint32_t& hi) {
    lo = ((zb & 0x0Fu) * 0x00010001u) | 0x64006400u;
    hi = ((zb & 0xF0u) * 0x00010001u) | 0x54005400u;
  }
};
template <> struct Dq<__nv_bfloat16> {
  // bf16 keeps 7 mantissa bits: every nibble is first moved to bits 0-3 of its half
  static __device__ __forceinline__ void run(uint32_t w, uint32_t bias_lo, uint32_t bias_hi, uint32_t (&a)[4]) {
    const uint32_t t0 = (w & 0x000F000Fu) | 0x43004300u;  // 128 + q
    const uint32_t t1 = ((w >> 4) & 0x000F000Fu) | 0x43004300u;
    const uint32_t t2 = ((w >> 8) & 0x000F000Fu) | 0x43004300u;
    const uint32_t t3 = ((w >> 12) & 0x000F000Fu) | 0x43004300u;
    asm("sub.bf16x2 %0, %1, %2;" : "=r"(a[0]) : "r"(t0), "r"(bias_lo));
    asm("sub.bf16x2 %0, %1, %2;" : "=r"(a[1]) : "r"(t1), "r"(bias_hi));
    asm("sub.bf16x2 %0, %1, %2;" : "=r"(a[2]) : "r"(t2), "r"(bias_lo));
    asm("sub.bf16x2 %0, %1, %2;" : "=r"(a[3]) : "r"(t3), "r"(bias_hi));
  }
  static __device__ __forceinline__ void bias(uint32_t zb, uint32_t& lo, uint32_t& hi) {
    lo = ((zb & 0x0Fu) * 0x00010001u) | 0x43004300u;
    hi = (((zb >> 4) & 0x0Fu) * 0x00010001u) | 0x43004300u;
  }
};

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ float2 s2_to_f2(uint32_t v, bool bf) {
  if (bf) return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(h);
}

// ---- the TMA-fed streaming kernel -------------------------------------------------------------
constexpr int kNC = 8;  // consumer warps
enum { kErrMnbTimeout = 301 };

__device__ __forceinline__ void consumer_barrier() {
  asm volatile("bar.sync 1, %0;" ::"r"(kNC * 32) : "memory");
}

template <typename T, int BLOCK, int NT>
__global__ void __launch_bounds__((kNC + 1) * 32)
mnb_tma_kernel(const T* __restrict__ A, const uint8_t* __restrict__ recs, T* __restrict__ Y, int M, int N, int K,
               int ntiles, int ksteps4, int G, int stages, int xrows, DeviceErrorSlot* err) {
  using RC = Rec<BLOCK>;
  constexpr int SPB = BLOCK / 16;
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  constexpr int UNIT = RC::kUnit;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + stages;
  int* flags = reinterpret_cast<int*>(empty + stages);
  unsigned char* buf = smem + 256;
  float* red = reinterpret_cast<float*>(buf + (size_t)stages * G * RC::kBytes);  // [kNC][NT][4][32]
  // staged activation rows (xrows > 0): xrows + 1 rows of kpad halves (columns >= K and the last row
  // zero), rows 16 bytes apart in bank order so the 8 row groups of a fragment load hit 32 banks
  unsigned char* xs = reinterpret_cast<unsigned char*>(red + kNC * NT * 4 * 32);
  const int kpad = ksteps4 * 64;
  const int xstride = kpad * 2 + 16;
  const bool stage_x = xrows > 0;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = (int)((int64_t)ntiles * blockIdx.x / gridDim.x);
  const int t1 = (int)((int64_t)ntiles * (blockIdx.x + 1) / gridDim.x);
  const int spt = (ksteps4 + G - 1) / G;  // stages per tile
  const int nst = (t1 - t0) * spt;
  const int m0 = blockIdx.y * 8 * NT;
  const int ksteps = K / 16;

  if (threadIdx.x == 0) {
    flags[0] = 0;
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kNC);
    }
    fence_mbarrier_init();
  }
  __syncthreads();
  if (warp == kNC) {
    if (lane == 0) {
      for (int i = 0; i < nst; ++i) {
        const int slot = i % stages;
        if (i >= stages && !mbar_wait(&empty[slot], ((i / stages) - 1) & 1)) {
          flags[0] = 1;
          break;
        }
        const int t = t0 + i / spt;
        const int ga = (i % spt) * G;
        const int n = min(G, ksteps4 - ga);
        const uint32_t bytes = (uint32_t)(n * RC::kBytes);
        mbar_arrive_expect_tx(&full[slot], bytes);
        bulk_g2s(buf + (size_t)slot * G * RC::kBytes, recs + ((size_t)t * ksteps4 + ga) * RC::kBytes, bytes,
                 &full[slot]);
      }
    }
    return;
  }

  // consumers: stage the activation rows of this column chunk (zero beyond K and beyond M) while
  // the producer's first copies are in flight
  if (stage_x) {
    const int wpr = kpad / 2;  // 32-bit words per row
    const int words = (xrows + 1) * wpr;
    for (int idx = threadIdx.x; idx < words; idx += kNC * 32) {
      const int r = idx / wpr, k = (idx - r * wpr) * 2;
      const int m = m0 + r;
      uint32_t v = 0;
      if (r < xrows && m < M && k < K) v = *reinterpret_cast<const uint32_t*>(A + (size_t)m * K + k);
      *reinterpret_cast<uint32_t*>(xs + (size_t)r * xstride + k * 2) = v;
    }
    consumer_barrier();
  }
  const int g = lane >> 2, c = lane & 3;
  const uint32_t* arow[NT];
  uint32_t amask[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int m = m0 + nt * 8 + g;
    if (stage_x) {
      // lanes without a token read the zero row: no predicate or mask in the loop
      const int r = m < M ? nt * 8 + g : xrows;  // m < M implies nt * 8 + g < xrows
      arow[nt] = reinterpret_cast<const uint32_t*>(xs + (size_t)r * xstride) + c;
      amask[nt] = 0xffffffffu;
    } else {
      amask[nt] = m < M ? 0xffffffffu : 0u;
      arow[nt] = reinterpret_cast<const uint32_t*>(A + (size_t)(m < M ? m : 0) * K) + c;
    }
  }
  float acc[NT][4], cb[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = cb[nt][e] = 0.f;

  bool alive = true;
  for (int i = 0; i < nst; ++i) {
    const int slot = i % stages;
    if (alive && !mbar_wait(&full[slot], (i / stages) & 1)) {
      flags[0] = 1;
      alive = false;
    }
    const int t = t0 + i / spt;
    const int ga = (i % spt) * G;
    const int n = alive ? min(G, ksteps4 - ga) : 0;
    const unsigned char* sb = buf + (size_t)slot * G * RC::kBytes;
    // records of this stage, in units of UNIT records per warp (a 128-block stays with one warp)
    for (int u = warp; u * UNIT < n; u += kNC) {
#pragma unroll
      for (int r = 0; r < UNIT; ++r) {
        const int q = u * UNIT + r;
        if (q >= n) break;
        const int gi = ga + q;
        const unsigned char* rec = sb + (size_t)q * RC::kBytes;
        uint32_t b[NT][8];
        if (stage_x) {
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const uint32_t* xr = arow[nt] + gi * 32;  // 64 halves per group
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              b[nt][2 * j] = xr[j * 8];
              b[nt][2 * j + 1] = xr[j * 8 + 4];
            }
          }
        } else {
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int s = gi * 4 + j;
              const int sc = s < ksteps ? s : 0;
              const uint32_t live = s < ksteps ? amask[nt] : 0u;
              b[nt][2 * j] = __ldg(arow[nt] + sc * 8) & live;
              b[nt][2 * j + 1] = __ldg(arow[nt] + sc * 8 + 4) & live;
            }
        }
        const uint4 w4 = *reinterpret_cast<const uint4*>(rec + lane * 16);
        const uint32_t words[4] = {w4.x, w4.y, w4.z, w4.w};
        uint32_t bias_lo = 0, bias_hi = 0;
        float2 scl = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const bool block_end = SPB <= 4 ? (j % SPB == SPB - 1) : (j == 3 && r == UNIT - 1);
          const int sl = SPB <= 4 ? j / SPB : 0;
          if (j % (SPB <= 4 ? SPB : 4) == 0) {  // parameters of the block this k-step belongs to
            const uint32_t sw = *reinterpret_cast<const uint32_t*>(rec + RC::kSOff + (sl * 8 + g) * 4);
            const uint32_t zb = rec[RC::kZOff + sl * 8 + g];
            scl = s2_to_f2(sw, BF);
            Dq<T>::bias(zb, bias_lo, bias_hi);
          }
          uint32_t a[4];
          Dq<T>::run(words[j], bias_lo, bias_hi, a);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma16816<T>(cb[nt], a, b[nt][2 * j], b[nt][2 * j + 1]);
          if (block_end) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              acc[nt][0] = fmaf(cb[nt][0], scl.x, acc[nt][0]);
              acc[nt][1] = fmaf(cb[nt][1], scl.x, acc[nt][1]);
              acc[nt][2] = fmaf(cb[nt][2], scl.y, acc[nt][2]);
              acc[nt][3] = fmaf(cb[nt][3], scl.y, acc[nt][3]);
              cb[nt][0] = cb[nt][1] = cb[nt][2] = cb[nt][3] = 0.f;
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    if (i % spt == spt - 1) {
      // tile finished: merge the consumers' partial sums
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          red[((warp * NT + nt) * 4 + e) * 32 + lane] = acc[nt][e];
          acc[nt][e] = 0.f;
        }
      consumer_barrier();
      if (warp == 0) {
        float sum[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kNC; ++w) v += red[((w * NT + nt) * 4 + e) * 32 + lane];
            sum[nt][e] = v;
          }
        const int n0 = t * 16 + g, n1 = n0 + 8;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int m = m0 + nt * 8 + 2 * c;
          if (m < M) {
            if (n0 < N) Y[(size_t)m * N + n0] = from_f<T>(sum[nt][0]);
            if (n1 < N) Y[(size_t)m * N + n1] = from_f<T>(sum[nt][2]);
          }
          if (m + 1 < M) {
            if (n0 < N) Y[(size_t)(m + 1) * N + n0] = from_f<T>(sum[nt][1]);
            if (n1 < N) Y[(size_t)(m + 1) * N + n1] = from_f<T>(sum[nt][3]);
          }
        }
      }
      consumer_barrier();
    }
  }
  if (flags[0] && threadIdx.x == 0) report_device_error(err, kErrMnbTimeout, blockIdx.x);
}

// ---- host side --------------------------------------------------------------------------------
MnbPacked mnb_packed_geometry(int64_t N, int64_t K, int block) {
  MnbPacked p{};
  p.N = N;
  p.K = K;
  p.block = block;
  p.nblocks_src = (K + block - 1) / block;
  p.ntiles = (N + 15) / 16;
  const int64_t unit = std::max<int64_t>(64, block);
  const int64_t kpad = ((K + unit - 1) / unit) * unit;
  p.ksteps4 = kpad / 64;
  p.record_bytes = mnb_record_bytes(block);
  p.bytes = (size_t)p.ntiles * p.ksteps4 * p.record_bytes;
  return p;
}

bool mnb_mma_supported(int dtype, int bits, int block, int64_t K) {
  return (dtype == kF16 || dtype == kBF16) && bits == 4 && K % 16 == 0 &&
         (block == 16 || block == 32 || block == 64 || block == 128);
}

namespace {
template <typename TS, int BLOCK>
cudaError_t prepack_t(const uint8_t* B, const void* scales, const uint8_t* zp, const MnbPacked& p, cudaStream_t st) {
  const int64_t work = (int64_t)p.ntiles * p.ksteps4 * std::max(128, Rec<BLOCK>::kBytes - 512);
  const int grid = (int)std::min<int64_t>((work + 255) / 256, 148 * 32);
  mnb_prepack_kernel<TS, BLOCK><<<grid, 256, 0, st>>>(B, static_cast<const TS*>(scales), zp, p);
  return cudaGetLastError();
}
template <typename TS>
cudaError_t prepack_b(const uint8_t* B, const void* scales, const uint8_t* zp, const MnbPacked& p, cudaStream_t st) {
  switch (p.block) {
    case 16: return prepack_t<TS, 16>(B, scales, zp, p, st);
    case 32: return prepack_t<TS, 32>(B, scales, zp, p, st);
    case 64: return prepack_t<TS, 64>(B, scales, zp, p, st);
    case 128: return prepack_t<TS, 128>(B, scales, zp, p, st);
  }
  return cudaErrorInvalidValue;
}

int num_sms() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}
}  // namespace

cudaError_t launch_mnb_prepack(const uint8_t* B, const void* scales, const uint8_t* zp, int scale_dtype,
                               const MnbPacked& p, cudaStream_t st) {
  if (scale_dtype == kF16) return prepack_b<__half>(B, scales, zp, p, st);
  if (scale_dtype == kBF16) return prepack_b<__nv_bfloat16>(B, scales, zp, p, st);
  return cudaErrorInvalidValue;
}

DeviceErrorSlot* device_error_slot();

namespace {
template <typename T, int BLOCK, int NT>
cudaError_t launch_tma_t(const void* A, const MnbPacked& p, void* Y, int64_t M, cudaStream_t st) {
  using RC = Rec<BLOCK>;
  const int G = 16;  // records per stage (~9.5 KB for block 32)
  const int stages = 4;
  // activation rows staged in shared memory when they fit in 64 KB (M = 1: K <= 16K)
  const int rows = (int)std::min<int64_t>(8 * NT, M);
  const size_t x_bytes = (size_t)(rows + 1) * (p.ksteps4 * 64 * 2 + 16);
  const int xrows = x_bytes <= 64 * 1024 ? rows : 0;
  const size_t smem = 256 + (size_t)stages * G * RC::kBytes + (size_t)kNC * NT * 4 * 32 * 4 + (xrows ? x_bytes : 0);
  auto kern = mnb_tma_kernel<T, BLOCK, NT>;
  static size_t configured = 0;  // per instantiation: the largest dynamic smem set so far
  if (smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured = smem;
  }
  static size_t occ_smem = 0;  // occupancy of the last smem size seen (one query per new size)
  static int per_sm = 1;
  if (smem != occ_smem) {
    int n = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, (kNC + 1) * 32, smem);
    if (e != cudaSuccess) return e;
    per_sm = std::max(1, n);
    occ_smem = smem;
  }
  const int64_t ctas = std::min<int64_t>(p.ntiles, (int64_t)per_sm * num_sms());
  dim3 grid((unsigned)ctas, (unsigned)((M + 8 * NT - 1) / (8 * NT)));
  kern<<<grid, (kNC + 1) * 32, smem, st>>>(static_cast<const T*>(A), static_cast<const uint8_t*>(p.w),
                                           static_cast<T*>(Y), (int)M, (int)p.N, (int)p.K, (int)p.ntiles,
                                           (int)p.ksteps4, G, stages, xrows, device_error_slot());
  return cudaGetLastError();
}

template <typename T, int BLOCK>
cudaError_t launch_nt(const void* A, const MnbPacked& p, void* Y, int64_t M, cudaStream_t st) {
  return M <= 8 ? launch_tma_t<T, BLOCK, 1>(A, p, Y, M, st) : launch_tma_t<T, BLOCK, 2>(A, p, Y, M, st);
}

template <typename T>
cudaError_t launch_b(const void* A, const MnbPacked& p, void* Y, int64_t M, cudaStream_t st) {
  switch (p.block) {
    case 16: return launch_nt<T, 16>(A, p, Y, M, st);
    case 32: return launch_nt<T, 32>(A, p, Y, M, st);
    case 64: return launch_nt<T, 64>(A, p, Y, M, st);
    case 128: return launch_nt<T, 128>(A, p, Y, M, st);
  }
  return cudaErrorInvalidValue;
}
}  // namespace

cudaError_t launch_mnb_packed(const void* A, const MnbPacked& p, void* Y, int dtype, int64_t M, cudaStream_t st) {
  if (M == 0) return cudaSuccess;
  if (dtype == kF16) return launch_b<__half>(A, p, Y, M, st);
  if (dtype == kBF16) return launch_b<__nv_bfloat16>(A, p, Y, M, st);
  return cudaErrorInvalidValue;
}

}  // namespace b200ep
