// MatMulNBits for many rows (prefill, M > 16) on the 5th-generation tensor cores: tcgen05.mma with
// the accumulator in tensor memory (reference: the fp16 prefill GEMM of quant.rs:540-601 and the
// quantised matmul of matmulnbits_op, quant.rs:986-1130).
//
// One CTA computes a (128 or 256) x 128 tile of Y = A . W^T, looping over K in 64-wide stages:
//   warp 0 (one lane)  TMA: the A tile(s) [128 rows x 64 k] through a 2-D tensor map with 128-byte
//                      swizzle into a ring of 3 stages (two row sub-tiles share each B tile when
//                      M > 128, halving the dequantisation per flop);
//   warp 2 (one lane)  the eight 16-row int4 group records of the W tile for each stage (1-D bulk
//                      copies from the prepacked stream) into a separate, deeper record ring (8, or
//                      4 with two sub-tiles), started before the wait for the previous kernel;
//   warps 3..18        dequantise the records (two warps per record, two 16-k steps each) into
//                      two B tiles [128 rows x 64 k] of the I/O dtype in the same 128-byte swizzled
//                      K-major layout, written with stmatrix straight from the fragment registers:
//                      hi = (q - z) * scale rounded once, lo = the rounding residual (one fused
//                      multiply-add), so hi + lo is the fp32 dequantised weight; fence them to the
//                      async proxy and arrive;
//   warp 1 (one lane)  issues tcgen05.mma.kind::f16 (128 x 128 x 16, fp32 in TMEM: hi and lo per
//                      16-k step and row sub-tile) and commits them to the stage's "empty" barrier,
//                      which frees the stage;
//   warps 3..18        finally read the accumulators with tcgen05.ld (a warp reads its 32 TMEM
//                      lanes; the four warps of a lane quarter split the columns) and store Y.
// CTAs along x cover the M tiles of one W tile, so the W tile is read from HBM once and the other
// M tiles find it in L2.  Every mbarrier wait is bounded (timeout -> device error word).
// (A persistent stream-K form — one CTA per SM sharing the (tile, 64-k stage) units, cut tiles
// summed from fp32 partials by their last contributor — measured slower on B200 at every prefill
// shape tried: the per-piece epilogue serialises the TMEM accumulator and the weight slabs lose
// their L2 reuse across concurrent CTAs.)
#include <cuda.h>
#include <cstdlib>

#include <algorithm>
#include <string>

#include "../common.cuh"
#include "kernels.h"
#include "mnb_mma.h"

namespace b200ep {

DeviceErrorSlot* device_error_slot();

namespace {

constexpr int kTM = 128, kTK = 64;
constexpr int kDeq = 16;      // dequantising (and epilogue) warps: 3 .. 3 + kDeq - 1 (8 or 16)
constexpr int kGThreads = (3 + kDeq) * 32;
enum { kErrGemmTimeout = 303 };
constexpr int kCost256x256 = 205;  // relative CTA time of a 256 x 256 tile (128 x 128 = 100)

template <int BLOCK>
struct GRec {  // the record geometry of mnb_mma.cu (kept in sync by mnb_record_bytes)
  static constexpr int kSlots = BLOCK >= 64 ? 1 : 64 / BLOCK;
  static constexpr int kSOff = 512;
  static constexpr int kZOff = 512 + kSlots * 32;
  static constexpr int kBytes = 512 + ((kSlots * 40 + 15) / 16) * 16;
};

// Tile geometry: MSUB 128-row sub-tiles of A share every dequantised B tile of TN (128 or 256)
// weight rows; the accumulators take MSUB x TN TMEM columns (at most 512).
template <int MSUB, int TN>
struct GemmSmem {
  static constexpr int kStages = TN == 256 ? 2 : 3;             // A / B tile ring
  static constexpr int kRPS = TN / 16;                          // weight records per stage
  static constexpr int kRS = TN == 256 ? 2 : MSUB == 1 ? 8 : 4; // weight-record ring depth
  static constexpr int kATile = kTM * kTK * 2;                  // 16 KB
  static constexpr int kA = 0;                                  // [stages][MSUB][128 x 64]
  static constexpr int kB = kA + kStages * MSUB * kATile;       // [stages][hi, lo][TN x 64]
  static constexpr int kBTile = TN * kTK * 2;
  static constexpr int kRec = kB + kStages * 2 * kBTile;        // [record stages][kRPS records]
  static constexpr int kRecStage = kRPS * 704;                  // largest record (block 16) x kRPS
  static constexpr int kBar = kRec + kRS * kRecStage;           // full, bready, empty, rfull, rempty, acc
  static constexpr int kTmemSlot = kBar + (3 * kStages + 2 * kRS + 1) * 8;
  static constexpr int kTotal = kTmemSlot + 16 + 1024;          // + alignment slack
  static_assert(MSUB * TN <= 512, "TMEM holds 512 fp32 columns");
  static_assert(kTotal <= 232448, "shared memory per CTA");
};

__device__ __forceinline__ uint64_t umma_desc(uint32_t smem_byte_addr) {
  // K-major, 128-byte swizzle: 8-row groups 1024 bytes apart (SBO), LBO unused (1), version 1
  uint64_t d = 0;
  d |= (uint64_t)((smem_byte_addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

template <typename T, int TN>
__device__ __forceinline__ uint32_t idesc_f16() {
  constexpr uint32_t fmt = std::is_same<T, __half>::value ? 0u : 1u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(TN >> 3) << 17) | ((uint32_t)(kTM >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// (a & b) | c
__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// 8 weights of one lane for k-step word w: rows g / g+8 at k {2c, 2c+1} and {2c+8, 2c+9}, as
// (q - z) * scale in T (pairs of the same row in one 32-bit word)
template <typename T>
__device__ __forceinline__ void dequant8(uint32_t w, uint32_t zr, uint32_t sg2, uint32_t sh2, uint32_t (&o)[4],
                                         uint32_t (&lo)[4]) {
  uint32_t t[4], blo, bhi;
  if constexpr (std::is_same<T, __half>::value) {
    const uint32_t w8 = w >> 8;
    t[0] = lop_and_or(w, 0x000F000Fu, 0x64006400u);
    t[1] = lop_and_or(w, 0x00F000F0u, 0x54005400u);
    t[2] = lop_and_or(w8, 0x000F000Fu, 0x64006400u);
    t[3] = lop_and_or(w8, 0x00F000F0u, 0x54005400u);
    blo = lop_and_or(zr, 0x000F000Fu, 0x64006400u);
    bhi = lop_and_or(zr, 0x00F000F0u, 0x54005400u);
    uint32_t q[4];
    asm("sub.f16x2 %0, %1, %2;" : "=r"(q[0]) : "r"(t[0]), "r"(blo));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(q[1]) : "r"(t[1]), "r"(bhi));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(q[2]) : "r"(t[2]), "r"(blo));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(q[3]) : "r"(t[3]), "r"(bhi));
    const uint32_t sc[4] = {sg2, sh2, sg2, sh2};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[i]) : "r"(q[i]), "r"(sc[i]));
      asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(lo[i]) : "r"(q[i]), "r"(sc[i]), "r"(o[i] ^ 0x80008000u));
    }
  } else {
    t[0] = lop_and_or(w, 0x000F000Fu, 0x43004300u);
    t[1] = lop_and_or(w >> 4, 0x000F000Fu, 0x43004300u);
    t[2] = lop_and_or(w >> 8, 0x000F000Fu, 0x43004300u);
    t[3] = lop_and_or(w >> 12, 0x000F000Fu, 0x43004300u);
    blo = lop_and_or(zr, 0x000F000Fu, 0x43004300u);
    bhi = lop_and_or(zr >> 4, 0x000F000Fu, 0x43004300u);
    uint32_t q[4];
    asm("sub.bf16x2 %0, %1, %2;" : "=r"(q[0]) : "r"(t[0]), "r"(blo));
    asm("sub.bf16x2 %0, %1, %2;" : "=r"(q[1]) : "r"(t[1]), "r"(bhi));
    asm("sub.bf16x2 %0, %1, %2;" : "=r"(q[2]) : "r"(t[2]), "r"(blo));
    asm("sub.bf16x2 %0, %1, %2;" : "=r"(q[3]) : "r"(t[3]), "r"(bhi));
    const uint32_t sc[4] = {sg2, sh2, sg2, sh2};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(o[i]) : "r"(q[i]), "r"(sc[i]));
      asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(lo[i]) : "r"(q[i]), "r"(sc[i]), "r"(o[i] ^ 0x80008000u));
    }
  }
}

// byte offset of element (row, k) in a 128 x 64 K-major tile with 128-byte swizzle
__device__ __forceinline__ uint32_t sw128(int row, int k) {
  return (uint32_t)(row * 128 + ((((k >> 3) ^ (row & 7)) & 7) << 4) + (k & 7) * 2);
}

// four 8 x 8 b16 matrices from mma fragment registers into shared memory rows (one 16-byte row
// segment per lane address: lanes 8m .. 8m + 7 give the rows of matrix m)
__device__ __forceinline__ void stsm_x4(uint32_t addr, const uint32_t (&r)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}

template <typename T, int BLOCK, int MSUB, int TN>
__global__ void __launch_bounds__(kGThreads, 1)
mnb_gemm_kernel(const __grid_constant__ CUtensorMap amap, const uint8_t* __restrict__ recs, T* __restrict__ Y,
                int M, int N, int ntiles, int ksteps4, DeviceErrorSlot* err) {
  using RC = GRec<BLOCK>;
  using GemmSmem = b200ep::GemmSmem<MSUB, TN>;
  constexpr int kRStages = GemmSmem::kRS;
  constexpr int kGStages = GemmSmem::kStages;
  constexpr int kTN = TN;
  constexpr int kRPS = GemmSmem::kRPS;
  constexpr int SPB = BLOCK / 16;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + GemmSmem::kBar);
  uint64_t* bready = full + kGStages;
  uint64_t* empty = bready + kGStages;
  uint64_t* rfull = empty + kGStages;
  uint64_t* rempty = rfull + kRStages;
  uint64_t* accbar = rempty + kRStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + GemmSmem::kTmemSlot);
  int* flag = reinterpret_cast<int*>(sm + GemmSmem::kTmemSlot + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kTM * MSUB, n0 = blockIdx.y * kTN;
  const int tile0 = n0 / 16;
  const int nst = ksteps4;  // stages: one 64-k group each

  if (threadIdx.x == 0) {
    *flag = 0;
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&bready[s], kDeq);
      mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < kRStages; ++r) {
      mbar_init(&rfull[r], 1);
      mbar_init(&rempty[r], kDeq);
    }
    mbar_init(accbar, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTN * MSUB));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  // Warp 2 streams weights (constants) at once; the other roles wait for the previous kernel
  // (A is its output; Y may still be read by it)
  if (warp != 2) {
    pdl_wait();
    pdl_trigger();
  }
  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < nst; ++i) {
        const int s = i % kGStages;
        if (i >= kGStages && !mbar_wait(&empty[s], ((i / kGStages) - 1) & 1)) {
          *flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], (uint32_t)(MSUB * GemmSmem::kATile));
        for (int u = 0; u < MSUB; ++u)
          tma_load_2d(sm + GemmSmem::kA + (s * MSUB + u) * GemmSmem::kATile, &amap, i * kTK, m0 + u * kTM, &full[s]);
      }
    }
  } else if (warp == 2) {
    if (lane == 0) {
      int nrec = 0;
      for (int j = 0; j < kRPS; ++j) nrec += tile0 + j < ntiles;
      for (int i = 0; i < nst; ++i) {
        const int r = i % kRStages;
        if (i >= kRStages && !mbar_wait(&rempty[r], ((i / kRStages) - 1) & 1)) {
          *flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&rfull[r], (uint32_t)(nrec * RC::kBytes));
        for (int j = 0; j < kRPS; ++j)
          if (tile0 + j < ntiles)
            bulk_g2s(sm + GemmSmem::kRec + r * GemmSmem::kRecStage + j * RC::kBytes,
                     recs + ((size_t)(tile0 + j) * ksteps4 + i) * RC::kBytes, RC::kBytes, &rfull[r]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16<T, TN>();
      bool alive = true;
      for (int i = 0; i < nst && alive; ++i) {
        const int s = i % kGStages;
        if (!mbar_wait(&full[s], (i / kGStages) & 1) || !mbar_wait(&bready[s], (i / kGStages) & 1)) {  // A, B
          *flag = 1;
          alive = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a0 = smem_u32(sm + GemmSmem::kA + s * MSUB * GemmSmem::kATile);
        const uint32_t b0 = smem_u32(sm + GemmSmem::kB + s * 2 * GemmSmem::kBTile);
#pragma unroll
        for (int kk = 0; kk < kTK / 16; ++kk)
#pragma unroll
          for (int u = 0; u < MSUB; ++u)  // row sub-tile u accumulates in TMEM columns [u * 128, u * 128 + 128)
#pragma unroll
            for (int part = 0; part < 2; ++part) {  // B.hi then B.lo
              const uint64_t ad = umma_desc(a0 + u * GemmSmem::kATile + kk * 32);
              const uint64_t bd = umma_desc(b0 + part * GemmSmem::kBTile + kk * 32);
              const uint32_t acc = (i > 0 || kk > 0 || part > 0) ? 1u : 0u;
              asm volatile(
                  "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                  "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(
                      tmem + (uint32_t)(u * kTN)),
                  "l"(ad), "l"(bd), "r"(idesc), "r"(acc), "r"(0u)
                  : "memory");
            }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&empty[s]))
                     : "memory");
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(accbar))
                   : "memory");
    }
    __syncwarp();
  } else {
    // warps 3 .. 3 + kDeq - 1: kDeq / kRPS warps per record, each dequantising 4 / (kDeq / kRPS)
    // of its k-steps per stage, then the epilogue
    constexpr int kDPR = kDeq / kRPS;  // warps per record
    static_assert(kDPR == 1 || kDPR == 2, "one or two dequantising warps per record");
    constexpr int kSPW = 4 / kDPR;  // k-steps per warp
    const int dw = warp - 3;
    const int j = dw / kDPR, st0 = (dw % kDPR) * kSPW;
    // stmatrix row address of this lane: matrix m = lane / 8 holds rows (m & 1) * 8 .. + 7 of the
    // record and k (m >> 1) * 8 .. + 7 of the k-step (the order of the mma A fragment registers)
    const int srow = j * 16 + ((lane >> 3) & 1) * 8 + (lane & 7), skh = (lane >> 4) * 8;
    const int g = lane >> 2;
    bool alive = true;
    for (int i = 0; i < nst; ++i) {
      const int s = i % kGStages, rr = i % kRStages;
      // the records of stage i, and a free B slot (the MMAs of stage i - kGStages completed)
      if (alive && !mbar_wait(&rfull[rr], (i / kRStages) & 1)) {
        *flag = 1;
        alive = false;
      }
      if (alive && i >= kGStages && !mbar_wait(&empty[s], ((i / kGStages) - 1) & 1)) {
        *flag = 1;
        alive = false;
      }
      unsigned char* bt = sm + GemmSmem::kB + s * 2 * GemmSmem::kBTile;
      unsigned char* bl = bt + GemmSmem::kBTile;
      const unsigned char* rs = sm + GemmSmem::kRec + rr * GemmSmem::kRecStage;
      const bool have = alive && tile0 + j < ntiles;
      const unsigned char* rec = rs + j * RC::kBytes;
      uint32_t words[kSPW];
#pragma unroll
      for (int u = 0; u < kSPW; ++u) words[u] = 0u;
      if (have) {
        if constexpr (kSPW == 4) {
          const uint4 w4 = *reinterpret_cast<const uint4*>(rec + lane * 16);
          words[0] = w4.x, words[1] = w4.y, words[2] = w4.z, words[3] = w4.w;
        } else {
          const uint2 w2 = *reinterpret_cast<const uint2*>(rec + lane * 16 + st0 * 4);
          words[0] = w2.x, words[1] = w2.y;
        }
      }
#pragma unroll
      for (int u = 0; u < kSPW; ++u) {
        const int st = st0 + u;
        const int sl = SPB <= 4 ? st / SPB : 0;
        uint32_t sw = 0, zr = 0;
        if (have) {
          sw = *reinterpret_cast<const uint32_t*>(rec + RC::kSOff + (g * RC::kSlots + sl) * 4);
          zr = __byte_perm((uint32_t)rec[RC::kZOff + g * RC::kSlots + sl], 0, 0x4040);
        }
        const uint32_t sg2 = __byte_perm(sw, 0, 0x1010), sh2 = __byte_perm(sw, 0, 0x3232);
        uint32_t o[4], lo[4];
        dequant8<T>(words[u], zr, sg2, sh2, o, lo);
        if (!have) o[0] = o[1] = o[2] = o[3] = lo[0] = lo[1] = lo[2] = lo[3] = 0u;
        const int kk = st * 16 + skh;
        stsm_x4(smem_u32(bt + sw128(srow, kk)), o);
        stsm_x4(smem_u32(bl + sw128(srow, kk)), lo);
      }
      // generic-proxy writes -> visible to the tensor core's (async proxy) reads
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bready[s]);
        mbar_arrive(&rempty[rr]);  // this warp's records of the slot are consumed
      }
    }
    // epilogue: warp w reads TMEM lanes 32 * (w % 4) .. + 31 (rows of the tile)
    if (!mbar_wait(accbar, 0)) *flag = 1;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // warp w reads TMEM lanes 32 * (w % 4) .. + 31; the kDeq / 4 warps of a lane quarter split the
    // (MSUB sub-tiles x 128) accumulator columns
    const int q = warp & 3, part = dw / 4, nparts = kDeq / 4;
    constexpr int kCols = kTN * MSUB;
#pragma unroll 1
    for (int ca = part * (kCols / nparts); ca < (part + 1) * (kCols / nparts); ca += 32) {
      const int u = ca / kTN, cc = ca % kTN;
      const int row = m0 + u * kTM + q * 32 + lane;
      uint32_t v[32];
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)ca;
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
          "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
            "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),
            "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
            "=r"(v[30]), "=r"(v[31])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (row < M) {
        T* yr = Y + (size_t)row * N + n0 + cc;
        const int ncol = min(32, N - (n0 + cc));
        if (ncol == 32 && (N % 8) == 0) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 pk;
            T* h = reinterpret_cast<T*>(&pk);
#pragma unroll
            for (int u = 0; u < 8; ++u) h[u] = from_f<T>(__uint_as_float(v[e + u]));
            *reinterpret_cast<uint4*>(yr + e) = pk;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e)  // constant indices keep v[] in registers
            if (e < ncol) yr[e] = from_f<T>(__uint_as_float(v[e]));
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTN * MSUB));
  }
  if (*flag && threadIdx.x == 0) report_device_error(err, kErrGemmTimeout, blockIdx.x);
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  }
  return fn;
}

template <typename T, int BLOCK, int MSUB, int TN>
cudaError_t gemm_t(const void* A, const MnbPacked& p, void* Y, int64_t M, cudaStream_t st) {
  EncodeTiled enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)p.K, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)p.K * 2};
  const cuuint32_t box[2] = {kTK, kTM};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (enc(&map, dt, 2, const_cast<void*>(A), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  auto kern = mnb_gemm_kernel<T, BLOCK, MSUB, TN>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmSmem<MSUB, TN>::kTotal);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  dim3 grid((unsigned)((M + kTM * MSUB - 1) / (kTM * MSUB)), (unsigned)((p.N + TN - 1) / TN));
  return launch_k(kern, grid, dim3(kGThreads), (size_t)GemmSmem<MSUB, TN>::kTotal, st, map,
                  static_cast<const uint8_t*>(p.w), static_cast<T*>(Y), (int)M, (int)p.N, (int)p.ntiles,
                  (int)p.ksteps4, device_error_slot());
}

// Tile shape per launch.  256-row CTAs dequantise each weight tile once for twice the MMAs; 256-
// column weight tiles halve the A-operand shared-memory reads per flop (a 128 x 128 x 16 MMA
// needs the whole shared-memory bandwidth; 128 x 256 x 16 leaves a quarter for the dequantised
// writes).  Relative CTA times measured on B200 over prefill shapes: 128x128 : 256x128 : 256x256 =
// 1 : 1.35 : 2.05; the choice minimises whole waves of 148 CTAs times that cost.
// ONNXRUNTIME_EP_B200_GEMM_TILE=128x128|256x128|256x256 forces one.
int gemm_tile(int64_t M, int64_t N) {
  static const int forced = [] {
    const char* e = std::getenv("ONNXRUNTIME_EP_B200_GEMM_TILE");
    if (!e) return 0;
    const std::string v(e);
    return v == "128x128" ? 1 : v == "256x128" ? 2 : v == "256x256" ? 3 : 0;
  }();
  if (forced) return forced;
  if (M <= kTM) return 1;
  auto waves = [&](int64_t rows, int64_t cols) {
    return ((M + rows - 1) / rows * ((N + cols - 1) / cols) + 147) / 148;
  };
  const int64_t c1 = waves(128, 128) * 100, c2 = waves(256, 128) * 135, c3 = waves(256, 256) * kCost256x256;
  return c3 <= c2 && c3 <= c1 ? 3 : c2 <= c1 ? 2 : 1;
}

template <typename T, int BLOCK>
cudaError_t gemm_m(const void* A, const MnbPacked& p, void* Y, int64_t M, cudaStream_t st) {
  switch (gemm_tile(M, p.N)) {
    case 3: return gemm_t<T, BLOCK, 2, 256>(A, p, Y, M, st);
    case 2: return gemm_t<T, BLOCK, 2, 128>(A, p, Y, M, st);
    default: return gemm_t<T, BLOCK, 1, 128>(A, p, Y, M, st);
  }
}

template <typename T>
cudaError_t gemm_b(const void* A, const MnbPacked& p, void* Y, int64_t M, cudaStream_t st) {
  switch (p.block) {
    case 16: return gemm_m<T, 16>(A, p, Y, M, st);
    case 32: return gemm_m<T, 32>(A, p, Y, M, st);
    case 64: return gemm_m<T, 64>(A, p, Y, M, st);
    case 128: return gemm_m<T, 128>(A, p, Y, M, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

// Rows from which the tcgen05 GEMM takes over from the GEMV (which runs 16-row chunks as grid rows,
// each re-streaming the weights).  Measured on B200 (fp16, block 32): at 24 and 32 rows the
// chunked GEMV is faster at every Llama-3-8B / 70B projection shape (down_proj K 14336: 58 us
// against 174 us, whose 32 weight tiles under-fill the GEMM's grid), at 48 rows the two are mixed,
// at 64 the GEMM wins.  ONNXRUNTIME_EP_B200_GEMM_MIN_ROWS overrides it (at least 17).
int64_t gemm_min_rows() {
  static const int64_t v = [] {
    const char* e = std::getenv("ONNXRUNTIME_EP_B200_GEMM_MIN_ROWS");
    const long long n = e ? std::atoll(e) : 0;
    return n > 16 ? (int64_t)n : (int64_t)33;
  }();
  return v;
}

bool mnb_gemm_supported(int64_t M, int64_t K, const void* A) {
  return M >= gemm_min_rows() && K % 16 == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0 && encode_fn() != nullptr;
}

cudaError_t launch_mnb_gemm(const void* A, const MnbPacked& p, void* Y, int dtype, int64_t M, cudaStream_t st) {
  if (M == 0) return cudaSuccess;
  if (dtype == kF16) return gemm_b<__half>(A, p, Y, M, st);
  if (dtype == kBF16) return gemm_b<__nv_bfloat16>(A, p, Y, M, st);
  return cudaErrorInvalidValue;
}

}  // namespace b200ep
