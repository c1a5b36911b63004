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
//   then, per row pair g and quantisation block the record covers (slot): the scales of rows g
//   and g+8 as one half2 / bf162 ([g][slot], so a lane loads all its slots at once), then their
//   zero points as one byte ([g][slot], row g + 8 in the high nibble); padded to 16 bytes.  Block 32: 512 + 80 = 592 bytes per 512 weight bytes, the same overhead
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
  static constexpr int kSOff = 512;                            // uint32 scales[8][slot]
  static constexpr int kZOff = 512 + kSlots * 32;              // uint8  zps[8][slot]
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
    const int g = idx / RC::kSlots, slot = idx % RC::kSlots;
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
// (a & b) | c as one LOP3.  The mask and magic constants live in registers (DqConst, built from a
// kernel argument the compiler cannot fold): with two immediates the and/or pair costs two
// integer-pipe instructions instead of one.
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

struct DqConst {
  uint32_t m0, m1, c0, c1;  // nibble masks 0x000F000F / 0x00F000F0 and the dtype's magic exponents
};

template <typename T> struct Dq;
template <> struct Dq<__half> {
  static __device__ __forceinline__ DqConst consts(uint32_t zero) {
    return DqConst{0x000F000Fu | zero, 0x00F000F0u | zero, 0x64006400u | zero, 0x54005400u | zero};
  }
  // (w & 0x000F000F) | 0x6400 -> 1024 + q; (w & 0x00F000F0) | 0x5400 -> 64 + q; exact subtract
  static __device__ __forceinline__ void run(uint32_t w, uint32_t bias_lo, uint32_t bias_hi, const DqConst& k,
                                             uint32_t (&a)[4]) {
    const uint32_t w8 = w >> 8;
    const uint32_t t0 = and_or(w, k.m0, k.c0);   // rows g,   k 2c / 2c+1
    const uint32_t t1 = and_or(w, k.m1, k.c1);   // rows g+8, k 2c / 2c+1
    const uint32_t t2 = and_or(w8, k.m0, k.c0);  // rows g,   k 2c+8 / 2c+9
    const uint32_t t3 = and_or(w8, k.m1, k.c1);  // rows g+8, k 2c+8 / 2c+9
    asm("sub.f16x2 %0, %1, %2;" : "=r"(a[0]) : "r"(t0), "r"(bias_lo));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(a[1]) : "r"(t1), "r"(bias_hi));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(a[2]) : "r"(t2), "r"(bias_lo));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(a[3]) : "r"(t3), "r"(bias_hi));
  }
  // zr = the zero-point byte (z_g | z_{g+8} << 4) in bytes 0 and 2
  // bias_lo = (1024 + z_g) in both halves, bias_hi = (64 + z_{g+8}) in both halves
  static __device__ __forceinline__ void bias(uint32_t zr, const DqConst& k, uint32_t& lo, uint32_t& hi) {
    lo = and_or(zr, k.m0, k.c0);
    hi = and_or(zr, k.m1, k.c1);
  }
};
template <> struct Dq<__nv_bfloat16> {
  static __device__ __forceinline__ DqConst consts(uint32_t zero) {
    return DqConst{0x000F000Fu | zero, 0x000F000Fu | zero, 0x43004300u | zero, 0x43004300u | zero};
  }
  // bf16 keeps 7 mantissa bits: every nibble is first moved to bits 0-3 of its half (128 + q)
  static __device__ __forceinline__ void run(uint32_t w, uint32_t bias_lo, uint32_t bias_hi, const DqConst& k,
                                             uint32_t (&a)[4]) {
    const uint32_t t0 = and_or(w, k.m0, k.c0);
    const uint32_t t1 = and_or(w >> 4, k.m0, k.c0);
    const uint32_t t2 = and_or(w >> 8, k.m0, k.c0);
    const uint32_t t3 = and_or(w >> 12, k.m0, k.c0);
    asm("sub.bf16x2 %0, %1, %2;" : "=r"(a[0]) : "r"(t0), "r"(bias_lo));
    asm("sub.bf16x2 %0, %1, %2;" : "=r"(a[1]) : "r"(t1), "r"(bias_hi));
    asm("sub.bf16x2 %0, %1, %2;" : "=r"(a[2]) : "r"(t2), "r"(bias_lo));
    asm("sub.bf16x2 %0, %1, %2;" : "=r"(a[3]) : "r"(t3), "r"(bias_hi));
  }
  static __device__ __forceinline__ void bias(uint32_t zr, const DqConst& k, uint32_t& lo, uint32_t& hi) {
    lo = and_or(zr, k.m0, k.c0);
    hi = and_or(zr >> 4, k.m0, k.c0);
  }
};

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// d = a . b with a zero accumulator (the first k-step of a quantisation block)
template <typename T>
__device__ __forceinline__ void mma16816_z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
  } else {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
  }
}

__device__ __forceinline__ float2 s2_to_f2(uint32_t v, bool bf) {
  if (bf) return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(h);
}

// ---- the TMA-fed streaming kernel -------------------------------------------------------------
// Geometry of the streaming kernel.  The defaults are the measured best on B200; the macros let a
// build try other splits without editing the kernel.
#ifndef B200EP_MNB_WARPS
#define B200EP_MNB_WARPS 8
#endif
#ifndef B200EP_MNB_STAGE_RECORDS
#define B200EP_MNB_STAGE_RECORDS 32
#endif
#ifndef B200EP_MNB_CTAS_PER_SM
#define B200EP_MNB_CTAS_PER_SM 2
#endif
constexpr int kNC = B200EP_MNB_WARPS;  // consumer warps
constexpr int kMinCtas = B200EP_MNB_CTAS_PER_SM;  // CTAs per SM the ring depth is chosen for
constexpr int kMaxStages = 4; // ring stages (chosen per launch: 2..4)
// bytes of staged activation rows (else fragments are read from global memory, which costs several
// times the weight stream at 8-16 rows): up to 16 rows at K = 4096 or 4 rows at K = 14336 (the
// launch then runs one CTA per SM when two no longer fit)
constexpr size_t kXStageMax = 144 * 1024;
// records per stage (one bulk copy, ~19 KB for 32 x block 32); long streams of staged activations run
// twice as many per stage (kGLong), which halves the waits and releases per record
constexpr int kG = B200EP_MNB_STAGE_RECORDS;
constexpr int kGLong = 2 * kG;
constexpr int kXcStride = kG * 64 * 2 + 16;  // bytes per activation row of a stage chunk (padded)
enum { kErrMnbTimeout = 301 };

__device__ __forceinline__ int64_t lmin(int64_t a, int64_t b) { return a < b ? a : b; }

// Tile-major records [beg(c), beg(c + 1)) of CTA c: whole tiles, spread evenly.
struct RecSplit {
  int64_t R;  // records
  int G;      // CTAs
  int ks;     // records per tile
  __device__ __forceinline__ int64_t beg(int c) const { return c >= G ? R : ((R / ks) * c / G) * ks; }
};

template <int NC>
__device__ __forceinline__ void consumer_barrier() {
  asm volatile("bar.sync 1, %0;" ::"r"(NC * 32) : "memory");
}

template <int N>
__device__ __forceinline__ void lds_words(const unsigned char* p, uint32_t (&v)[N]) {
  if constexpr (N == 1) {
    v[0] = *reinterpret_cast<const uint32_t*>(p);
  } else if constexpr (N == 2) {
    const uint2 t = *reinterpret_cast<const uint2*>(p);
    v[0] = t.x, v[1] = t.y;
  } else {
    const uint4 t = *reinterpret_cast<const uint4*>(p);
    v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
  }
}

// Activation rows staged in shared memory in fragment order: per row and 64-k group, lane column
// c owns 8 consecutive words (its B fragments of the group's 4 k-steps: k 2c,2c+1 then 2c+8,2c+9
// of each k-step), so a lane loads a record's B operands with two 16-byte loads.
__device__ __forceinline__ int xperm_src_word(int w) {  // word within a 64-k group, staged order -> k order
  const int c = w >> 3, j = (w >> 1) & 3, h = w & 1;
  return j * 8 + h * 4 + c;
}

// Write 8 consecutive activations (k .. k+7 of one row, k % 8 == 0) into the fragment-order row.
__device__ __forceinline__ void xs_put(unsigned char* row, int k, uint4 v) {
  const int kw = k >> 1;                           // first source word of the chunk
  const int grp = kw & ~31, sw = kw & 31;          // sw = j*8 + h*4 (c = 0..3 follow)
  const int j = sw >> 3, h = (sw >> 2) & 1;
  uint32_t* dst = reinterpret_cast<uint32_t*>(row) + grp + 2 * j + h;
  dst[0] = v.x, dst[8] = v.y, dst[16] = v.z, dst[24] = v.w;
}

template <typename T>
__device__ __forceinline__ void unpack8(uint4 v, float (&f)[8]) {
  const T* h = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f<T>(h[i]);
}
template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 v;
  T* h = reinterpret_cast<T*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = from_f<T>(f[i]);
  return v;
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

enum { kErrArTimeout = 302 };

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Consumer side of the peer-memory all-reduce: wait until every source rank published `epoch`
// (bounded; a timeout records an error and proceeds), then x chunks are sums of the slots.
__device__ bool ar_wait(const MnbAr& ar, unsigned epoch, DeviceErrorSlot* err) {
  bool ok = true;
  if ((int)threadIdx.x < ar.world) {
    const unsigned* flag = reinterpret_cast<const unsigned*>(ar.mbox[ar.rank]) + threadIdx.x;
    uint32_t it = 0;
    while ((int)(ld_acquire_sys(flag) - epoch) < 0) {
      if (++it > (1u << 24)) {  // ~1 s of polling: the peer is gone
        report_device_error(err, kErrArTimeout, (int)threadIdx.x);
        ok = false;
        break;
      }
    }
  }
  return ok;
}

template <typename T>
__device__ __forceinline__ void ar_sum8(const MnbAr& ar, unsigned epoch, size_t elem, float (&f)[8]) {
  const char* base = ar.mbox[ar.rank] + kArFlagsBytes + (size_t)(epoch & 1) * ar.region_bytes + elem * sizeof(T);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = 0.f;
  for (int src = 0; src < ar.world; ++src) {
    float v[8];
    unpack8<T>(__ldcg(reinterpret_cast<const uint4*>(base + (size_t)src * ar.slot_bytes)), v);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] += v[i];
  }
  // the all-reduced activation is an I/O-dtype tensor
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f<T>(from_f<T>(f[i]));
}

// Fused producers of the staged activations (consumer threads only; ends before the caller's
// barrier).  Arithmetic follows the standalone kernels: SiLU(g) * u as in silu_mul_kernel, and the
// (skip) RMS norm as in rms_norm_kernel — fp32 sum of squares of the (unrounded) row, y =
// (t * inv) * gamma rounded once; the skip form writes the rounded sum t to pro.residual from the
// CTAs of column 0 (blockIdx.x == 0).  wsum: kNC floats of scratch for the per-warp partials.
template <typename T, int NC>
__device__ void stage_prologue(const MnbPro& pro, unsigned char* xs, int xstride, int kpad, int xrows, int m0,
                               int M, int K, float* wsum, DeviceErrorSlot* err) {
  const int tid = threadIdx.x, nthr = NC * 32;
  const int cpr = kpad / 8;
  // zero row (index xrows) for lanes without a token
  for (int kc = tid; kc < cpr; kc += nthr) xs_put(xs + (size_t)xrows * xstride, kc * 8, make_uint4(0, 0, 0, 0));
  if (pro.kind == kProSiluMul) {
    const T* gu = static_cast<const T*>(pro.x);
    for (int idx = tid; idx < xrows * cpr; idx += nthr) {
      const int r = idx / cpr, k = (idx - r * cpr) * 8;
      const int m = m0 + r;
      float f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (m < M && k < K) {
        float gf[8], uf[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(gu + (size_t)m * 2 * K + k), gf);
        unpack8<T>(*reinterpret_cast<const uint4*>(gu + (size_t)m * 2 * K + K + k), uf);
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = gf[i] / (1.f + __expf(-gf[i])) * uf[i];
      }
      xs_put(xs + (size_t)r * xstride, k, pack8<T>(f));
    }
    return;
  }
  const T* X = static_cast<const T*>(pro.x);
  const T* S = static_cast<const T*>(pro.skip);
  const T* G = static_cast<const T*>(pro.gamma);
  T* R = blockIdx.x == 0 ? static_cast<T*>(pro.residual) : nullptr;
  const bool skip = pro.kind == kProSkipRms;
  // x comes from the peer mailboxes (tensor-parallel partial sums) instead of X
  const bool from_ar = skip && pro.ar.world > 0;
  unsigned epoch = 0;
  if (from_ar) {
    epoch = __ldcg(pro.ar.ctrs);
    ar_wait(pro.ar, epoch, err);
    consumer_barrier<NC>();
  }
  auto load_x = [&](int m, int k, float (&t)[8]) {
    if (from_ar)
      ar_sum8<T>(pro.ar, epoch, (size_t)m * K + k, t);
    else
      unpack8<T>(*reinterpret_cast<const uint4*>(X + (size_t)m * K + k), t);
  };
  for (int r = 0; r < xrows; ++r) {
    const int m = m0 + r;
    if (m >= M) {
      for (int kc = tid; kc < cpr; kc += nthr) xs_put(xs + (size_t)r * xstride, kc * 8, make_uint4(0, 0, 0, 0));
      continue;
    }
    constexpr int kCh = 2;  // chunks of 8 a thread keeps in registers: one pass over x when kpad fits
    if (kpad <= kCh * 8 * nthr) {
      float t[kCh][8], gm[kCh][8], ss = 0.f;
#pragma unroll
      for (int j = 0; j < kCh; ++j) {
        const int k = (tid + j * nthr) * 8;
        if (k < K) {
          load_x(m, k, t[j]);
          unpack8<T>(*reinterpret_cast<const uint4*>(G + k), gm[j]);
          if (skip) {
            float sk[8];
            unpack8<T>(*reinterpret_cast<const uint4*>(S + (size_t)m * K + k), sk);
#pragma unroll
            for (int i = 0; i < 8; ++i) t[j][i] += sk[i];
            if (R) *reinterpret_cast<uint4*>(R + (size_t)m * K + k) = pack8<T>(t[j]);
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) ss = fmaf(t[j][i], t[j][i], ss);
        }
      }
      ss = warp_sum(ss);
      if ((tid & 31) == 0) wsum[tid >> 5] = ss;
      consumer_barrier<NC>();
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < NC; ++w) tot += wsum[w];
      const float inv = rsqrtf(tot / (float)K + pro.eps);
#pragma unroll
      for (int j = 0; j < kCh; ++j) {
        const int k = (tid + j * nthr) * 8;
        if (k < kpad) {
          float y[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) y[i] = k < K ? t[j][i] * inv * gm[j][i] : 0.f;
          xs_put(xs + (size_t)r * xstride, k, pack8<T>(y));
        }
      }
      consumer_barrier<NC>();  // wsum is reused by the next row
      continue;
    }
    float ss = 0.f;
    for (int kc = tid; kc * 8 < K; kc += nthr) {
      float t[8];
      load_x(m, kc * 8, t);
      if (skip) {
        float sk[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(S + (size_t)m * K + kc * 8), sk);
#pragma unroll
        for (int i = 0; i < 8; ++i) t[i] += sk[i];
        if (R) *reinterpret_cast<uint4*>(R + (size_t)m * K + kc * 8) = pack8<T>(t);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(t[i], t[i], ss);
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) wsum[tid >> 5] = ss;
    consumer_barrier<NC>();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < NC; ++w) tot += wsum[w];
    const float inv = rsqrtf(tot / (float)K + pro.eps);
    for (int kc = tid; kc < cpr; kc += nthr) {
      const int k = kc * 8;
      float y[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (k < K) {
        float t[8], gm[8];
        load_x(m, k, t);
        if (skip) {
          float sk[8];
          unpack8<T>(*reinterpret_cast<const uint4*>(S + (size_t)m * K + k), sk);
#pragma unroll
          for (int i = 0; i < 8; ++i) t[i] += sk[i];
        }
        unpack8<T>(*reinterpret_cast<const uint4*>(G + k), gm);
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = t[i] * inv * gm[i];
      }
      xs_put(xs + (size_t)r * xstride, k, pack8<T>(y));
    }
    consumer_barrier<NC>();  // wsum is reused by the next row
  }
}

// One unit (UNIT consecutive records of one warp): dequantise, MMA per k-step, scale per block.
//   wq: this lane's 16 weight bytes of the first record; pq: the first record (parameters)
//   xp: staged activation fragments of the first record (STAGED) — else ag/live/gi0 address the
//   activation rows in global memory.  PAIR = false when only even token columns exist (M == 1):
//   the odd-column accumulators are then left alone.
template <typename T, int BLOCK, int NT, int XM, bool PAIR>
__device__ __forceinline__ void mnb_unit(const unsigned char* wq, const unsigned char* pq,
                                         const unsigned char* const (&xp)[NT], const uint32_t* const (&ag)[NT],
                                         const uint32_t (&live)[NT], int gi0, int ksteps, int g,
                                         const DqConst& kq, float (&acc)[NT][4], uint32_t xc = 0) {
  using RC = Rec<BLOCK>;
  constexpr int SPB = BLOCK / 16;
  constexpr int SL = RC::kSlots;
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  float cb[NT][4];
#pragma unroll
  for (int r = 0; r < RC::kUnit; ++r) {
    uint32_t b[NT][8];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      if constexpr (XM == 2) {
        // row-major chunk of this stage: ldmatrix per k-step (matrices: tokens 0-7 / 8-15 x k 0-7 / 8-15)
        if (nt == 0) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t a = xc + (uint32_t)(r * 128 + j * 32);
            if constexpr (NT == 2) {
              asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                           : "=r"(b[0][2 * j]), "=r"(b[0][2 * j + 1]), "=r"(b[1][2 * j]), "=r"(b[1][2 * j + 1])
                           : "r"(a));
            } else {
              asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
                           : "=r"(b[0][2 * j]), "=r"(b[0][2 * j + 1])
                           : "r"(a));
            }
          }
#pragma unroll
          for (int q = 0; q < NT; ++q)
#pragma unroll
            for (int e = 0; e < 8; ++e) b[q][e] &= live[q];
        }
      } else if constexpr (XM == 1) {
        const uint4 lo = *reinterpret_cast<const uint4*>(xp[nt] + r * 128);
        const uint4 hi = *reinterpret_cast<const uint4*>(xp[nt] + r * 128 + 16);
        b[nt][0] = lo.x, b[nt][1] = lo.y, b[nt][2] = lo.z, b[nt][3] = lo.w;
        b[nt][4] = hi.x, b[nt][5] = hi.y, b[nt][6] = hi.z, b[nt][7] = hi.w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int s = (gi0 + r) * 4 + j;
          const int sc = s < ksteps ? s : 0;
          const uint32_t lv = s < ksteps ? live[nt] : 0u;
          b[nt][2 * j] = __ldg(ag[nt] + sc * 8) & lv;
          b[nt][2 * j + 1] = __ldg(ag[nt] + sc * 8 + 4) & lv;
        }
      }
    }
    const unsigned char* rec = pq + r * RC::kBytes;
    const uint4 w4 = *reinterpret_cast<const uint4*>(wq + r * RC::kBytes);
    const uint32_t words[4] = {w4.x, w4.y, w4.z, w4.w};
    uint32_t sw[SL];
    lds_words<SL>(rec + RC::kSOff + g * SL * 4, sw);
    const uint32_t zz = SL == 1 ? (uint32_t)rec[RC::kZOff + g]
                        : SL == 2 ? (uint32_t)*reinterpret_cast<const uint16_t*>(rec + RC::kZOff + g * 2)
                                  : *reinterpret_cast<const uint32_t*>(rec + RC::kZOff + g * 4);
    uint32_t bias_lo = 0, bias_hi = 0;
    float2 scl = make_float2(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bool block_start = SPB <= 4 ? (j % SPB == 0) : (j == 0 && r == 0);
      const bool block_end = SPB <= 4 ? (j % SPB == SPB - 1) : (j == 3 && r == RC::kUnit - 1);
      const int sl = SPB <= 4 ? j / SPB : 0;
      if (j % (SPB <= 4 ? SPB : 4) == 0) {  // parameters of the block this k-step belongs to
        scl = s2_to_f2(sw[sl], BF);
        Dq<T>::bias(__byte_perm(zz, 0, 0x4040 + 0x0101 * sl), kq, bias_lo, bias_hi);
      }
      uint32_t a[4];
      Dq<T>::run(words[j], bias_lo, bias_hi, kq, a);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        if (block_start)
          mma16816_z<T>(cb[nt], a, b[nt][2 * j], b[nt][2 * j + 1]);
        else
          mma16816<T>(cb[nt], a, b[nt][2 * j], b[nt][2 * j + 1]);
      }
      if (block_end) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          acc[nt][0] = fmaf(cb[nt][0], scl.x, acc[nt][0]);
          acc[nt][2] = fmaf(cb[nt][2], scl.y, acc[nt][2]);
          if (PAIR) {
            acc[nt][1] = fmaf(cb[nt][1], scl.x, acc[nt][1]);
            acc[nt][3] = fmaf(cb[nt][3], scl.y, acc[nt][3]);
          }
        }
      }
    }
  }
}

template <typename T, int BLOCK, int NT, bool PAIR, int NC, int G>
__global__ void __launch_bounds__((NC + 1) * 32, NC > kNC ? 1 : kMinCtas)
mnb_tma_kernel(const T* __restrict__ A, const uint8_t* __restrict__ recs, T* __restrict__ Y, int M, int N, int K,
               int ntiles, int ksteps4, int xrows, int xmode, uint32_t zero, int stages, MnbPro pro, MnbAr oar,
               DeviceErrorSlot* err) {
  using RC = Rec<BLOCK>;
  constexpr int UNIT = RC::kUnit;
  constexpr int PER = G / (NC * UNIT);   // units per warp per full stage
  static_assert(G % (NC * UNIT) == 0, "stage must split evenly");
  static_assert(G == kG || G == kGLong, "stage size");
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  int* flags = reinterpret_cast<int*>(empty + kMaxStages);
  unsigned char* buf = smem + 256;
  // ring stage: G records, then (xmode 2, G == kG only) the stage's k-range of the 8 NT activation rows,
  // row-major with rows kXcStride bytes apart (bulk-copied beside the records)
  const size_t rec_bytes = (size_t)G * RC::kBytes;
  const size_t stage_bytes = rec_bytes + (xmode == 2 ? (size_t)8 * NT * kXcStride : 0);
  float* red = reinterpret_cast<float*>(buf + (size_t)stages * stage_bytes);  // [2][NC][NT][4][32]
  // staged activation rows (xrows > 0): xrows + 1 rows (the last one zero) of kpad halves,
  // 16 bytes apart in bank order so the 8 row groups of a fragment load use all 32 banks
  unsigned char* xs = reinterpret_cast<unsigned char*>(red + 2 * NC * NT * 4 * 32);
  const int kpad = ksteps4 * 64;
  const int xstride = kpad * 2 + 16;
  const bool stage_x = xmode == 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const RecSplit part{(int64_t)ntiles * ksteps4, (int)gridDim.x, ksteps4};
  const int64_t rbeg = part.beg(blockIdx.x), rend = part.beg(blockIdx.x + 1);
  const int m0 = blockIdx.y * 8 * NT;
  const int vrows = min(8 * NT, M - m0);  // activation rows of this column chunk
  const int ksteps = K / 16;

  if (threadIdx.x == 0) {
    flags[0] = 0;
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NC);
    }
    fence_mbarrier_init();
  }
  __syncthreads();
  // the weight stream reads constants only and starts at once; the consumers wait for the previous
  // kernel before they read activations or write outputs
  if (warp == NC) {
    if (lane == 0) {
      // the CTA's records in stages of at most G that never cross a tile boundary
      int slot = 0;
      uint32_t phase = 0;
      int64_t r = rbeg;
      // xmode 2: the activation rows of a stage's k-range (64 k per record) are bulk-copied beside
      // its records.  They are the previous kernel's output, so the records of the first ring
      // stages go out at once and their activation chunks only after the wait for that kernel.
      auto copy_x = [&](int sl, int64_t rr, int n) {
        const int kr = (int)(rr - (rr / ksteps4) * ksteps4);
        unsigned char* sb = buf + (size_t)sl * stage_bytes;
        for (int row = 0; row < vrows; ++row)
          bulk_g2s(sb + rec_bytes + (size_t)row * kXcStride, A + (size_t)(m0 + row) * K + (size_t)kr * 64,
                   (uint32_t)(n * 128), &full[sl]);
      };
      bool waited = xmode != 2;
      int npend = 0;  // stages issued without their chunks: the first npend stages from rbeg
      auto flush = [&]() {
        pdl_wait();
        int64_t rr = rbeg;
        for (int j = 0; j < npend; ++j) {
          const int nn = (int)lmin(G, lmin(rend, (rr / ksteps4 + 1) * ksteps4) - rr);
          copy_x(j, rr, nn);
          rr += nn;
        }
        npend = 0;
        waited = true;
      };
      for (int i = 0; r < rend; ++i) {
        if (i >= stages && !waited) flush();  // before the ring wraps: the consumers need these chunks
        if (i >= stages && !mbar_wait(&empty[slot], phase ^ 1)) {
          flags[0] = 1;
          break;
        }
        const int64_t tile_end = (r / ksteps4 + 1) * ksteps4;
        const int n = (int)lmin(G, lmin(rend, tile_end) - r);
        const uint32_t bytes = (uint32_t)(n * RC::kBytes);
        unsigned char* sbuf = buf + (size_t)slot * stage_bytes;
        if (xmode == 2) {
          mbar_arrive_expect_tx(&full[slot], bytes + (uint32_t)(vrows * n * 128));
          if (waited)
            copy_x(slot, r, n);
          else  // i < stages here, so slot == i == npend
            ++npend;
        } else {
          mbar_arrive_expect_tx(&full[slot], bytes);
        }
        bulk_g2s(sbuf, recs + (size_t)r * RC::kBytes, bytes, &full[slot]);
        r += n;
        if (++slot == stages) slot = 0, phase ^= 1;
      }
      if (!waited) flush();
    }
    return;
  }

  // consumers: stage the activation rows of this column chunk while the first copies are in flight
  pdl_wait();
  pdl_trigger();
  // tensor-parallel partial output: this launch publishes epoch + 1 (see MnbAr)
  const unsigned oepoch = oar.world ? __ldcg(oar.ctrs) + 1 : 0;

  if (stage_x) {
    if (pro.kind == kProNone) {
      // 16-byte loads (8 k), each scattered to its 4 fragment-order words; K % 8 == 0 here
      const int cpr = kpad / 8;  // 16-byte chunks per row
      const int chunks = (xrows + 1) * cpr;
      for (int base = threadIdx.x; base < chunks; base += 4 * NC * 32) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int idx = base + u * NC * 32;
          const int r = idx / cpr, k = (idx - r * cpr) * 8;
          const int m = m0 + r;
          v[u] = make_uint4(0, 0, 0, 0);
          if (idx < chunks && r < xrows && m < M && k < K) v[u] = *reinterpret_cast<const uint4*>(A + (size_t)m * K + k);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int idx = base + u * NC * 32;
          if (idx < chunks) xs_put(xs + (size_t)(idx / cpr) * xstride, (idx % cpr) * 8, v[u]);
        }
      }
    } else {
      stage_prologue<T, NC>(pro, xs, xstride, kpad, xrows, m0, M, K, red + 2 * NC * NT * 4 * 32 - NC, err);
    }
    consumer_barrier<NC>();
  } else if (xmode == 2 && vrows < 8 * NT) {
    // rows without a token read zeros (the copies only ever write rows < vrows)
    const int per_row = kXcStride / 16;
    for (int s = 0; s < stages; ++s)
      for (int i = threadIdx.x; i < (8 * NT - vrows) * per_row; i += NC * 32)
        *reinterpret_cast<uint4*>(buf + (size_t)s * stage_bytes + rec_bytes +
                                  (size_t)(vrows + i / per_row) * kXcStride + (i % per_row) * 16) = make_uint4(0, 0, 0, 0);
    consumer_barrier<NC>();
  }
  const int g = lane >> 2, c = lane & 3;
  const unsigned char* xrow[NT];
  const uint32_t* arow[NT];
  uint32_t amask[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int m = m0 + nt * 8 + g;
    // lanes without a token read the zero row: no predicate or mask in the loop
    const int r = m < M ? nt * 8 + g : xrows;  // m < M implies nt * 8 + g < xrows
    xrow[nt] = xs + (size_t)r * xstride + c * 32;
    amask[nt] = m < M ? 0xffffffffu : 0u;
    arow[nt] = reinterpret_cast<const uint32_t*>(A + (size_t)(m < M ? m : 0) * K) + c;
  }
  const unsigned char* xzero = xs + (size_t)xrows * xstride + c * 32;
  const DqConst kq = Dq<T>::consts(zero);
  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;

  // per-warp bases: the warp's first record in stage 0 and its activation fragments
  const unsigned char* wrec = buf + (size_t)warp * UNIT * RC::kBytes + lane * 16;
  const unsigned char* wparam = buf + (size_t)warp * UNIT * RC::kBytes;
  bool alive = true;
  int slot = 0, tp = 0;
  uint32_t phase = 0;
  int t = (int)(rbeg / ksteps4), ga = (int)(rbeg - (int64_t)t * ksteps4);
  int gend = (int)lmin(rend - (int64_t)t * ksteps4, ksteps4);  // end of the segment
  while ((int64_t)t * ksteps4 + ga < rend) {
    if (alive && !mbar_wait(&full[slot], phase)) {
      flags[0] = 1;
      alive = false;
    }
    const int nplan = min(G, gend - ga);
    const int n = alive ? nplan : 0;
    const size_t soff = (size_t)slot * stage_bytes;
    if (xmode == 2) {
      // activation chunk of this stage: ldmatrix rows (token (lane / 16) * 8 + lane % 8, k half
      // (lane / 8) % 2) of the unit's records
      const uint32_t xc0 = smem_u32(buf + soff + rec_bytes) +
                           (uint32_t)((((lane >> 4) * 8 + (lane & 7)) * kXcStride) + ((lane >> 3) & 1) * 16);
#pragma unroll
      for (int pu = 0; pu < PER; ++pu) {
        const int q0 = (pu * NC + warp) * UNIT;
        const bool valid = q0 < n;
        const int q = valid ? q0 : 0;
        uint32_t live[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) live[nt] = valid ? 0xffffffffu : 0u;
        const unsigned char* xp[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) xp[nt] = nullptr;
        const unsigned char* r0 = buf + soff + (size_t)q * RC::kBytes;
        mnb_unit<T, BLOCK, NT, 2, PAIR>(r0 + lane * 16, r0, xp, arow, live, 0, ksteps, g, kq, acc,
                                        xc0 + (uint32_t)(q * 128));
      }
    } else if (stage_x && n == G) {
      // full stage: every address is a per-stage base plus a compile-time offset
      const int xoff = (ga + warp * UNIT) * 128;
#pragma unroll
      for (int pu = 0; pu < PER; ++pu) {
        const int qoff = pu * NC * UNIT;
        const unsigned char* xp[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) xp[nt] = xrow[nt] + xoff + qoff * 128;
        mnb_unit<T, BLOCK, NT, 1, PAIR>(wrec + soff + qoff * RC::kBytes, wparam + soff + qoff * RC::kBytes, xp,
                                     arow, amask, 0, ksteps, g, kq, acc);
      }
    } else {
      // short stage (or activations read from global memory): units past the end rerun the
      // stage's first unit against zero activations (finite parameters, contribution exactly 0)
#pragma unroll
      for (int pu = 0; pu < PER; ++pu) {
        const int q0 = (pu * NC + warp) * UNIT;
        const bool valid = q0 < n;
        const int q = valid ? q0 : 0;
        const unsigned char* xp[NT];
        uint32_t live[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          xp[nt] = (valid ? xrow[nt] : xzero) + (ga + q) * 128;
          live[nt] = valid ? amask[nt] : 0u;
        }
        const unsigned char* r0 = buf + soff + (size_t)q * RC::kBytes;
        if (stage_x)
          mnb_unit<T, BLOCK, NT, 1, PAIR>(r0 + lane * 16, r0, xp, arow, live, ga + q, ksteps, g, kq, acc);
        else
          mnb_unit<T, BLOCK, NT, 0, PAIR>(r0 + lane * 16, r0, xp, arow, live, ga + q, ksteps, g, kq, acc);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    if (++slot == stages) slot = 0, phase ^= 1;
    ga += nplan;
    if (ga >= gend) {
      // tile finished: merge the consumers' partial sums.  red is double-buffered by tile
      // parity, so one barrier per tile suffices (a buffer is rewritten only after the next
      // tile's barrier, which every warp reaches after finishing its part of this merge).  Thread
      // tid sums output row tid / 16, column tid % 16: a 1-token chunk spreads over all warps.
      // (Measured alternatives, both slower on B200: a barrier-free merge by the last warp to
      // arrive, which then does the whole reduction alone; and record-granular balancing inside
      // thread-block clusters with cut tiles summed through distributed shared memory — a
      // cluster launches only when a GPC frees enough slots at once, defeating the overlap with
      // the previous kernel.)
      float* rb = red + (size_t)(tp & 1) * NC * NT * 4 * 32;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (PAIR || !(e & 1)) rb[((warp * NT + nt) * 4 + e) * 32 + lane] = acc[nt][e];
          acc[nt][e] = 0.f;
        }
      consumer_barrier<NC>();
      // thread tid sums output row tid % 16 of token column tid / 16: a column's 16 rows are 16
      // lanes of one warp, so its outputs are one 32-byte store
      for (int tid = threadIdx.x; tid < 256; tid += NC * 32) {
        const int row = tid & 15, col = tid >> 4;
        const int m = m0 + col, n = t * 16 + row;
        const bool ok = col < 8 * NT && m < M && n < N;
        float v = 0.f;
        if (ok) {
          const int nt = col >> 3, cc = col & 7;
          const int e = (row >= 8 ? 2 : 0) + (cc & 1);
          const int ln = (row & 7) * 4 + (cc >> 1);
#pragma unroll
          for (int w = 0; w < NC; ++w) v += rb[((w * NT + nt) * 4 + e) * 32 + ln];
        }
        if (!pro.swiglu) {
          if (ok) Y[(size_t)m * N + n] = from_f<T>(v);
        } else {
          // rows 8..15 of the tile are the up projections of rows 0..7 (lane + 8 of this warp);
          // both rounded to T first, as the separate SiLU * up kernel reads them
          const float u = __shfl_down_sync(0xffffffffu, v, 8);
          if (ok && row < 8) {
            const float gf = round_through<T>(v), uf = round_through<T>(u);
            Y[(size_t)m * (N / 2) + t * 8 + row] = from_f<T>(gf / (1.f + __expf(-gf)) * uf);
          }
        }
      }
      ++tp;
      ++t;
      ga = 0;
      gend = (int)lmin(rend - (int64_t)t * ksteps4, ksteps4);
    }
  }
  if (flags[0] && threadIdx.x == 0) report_device_error(err, kErrMnbTimeout, blockIdx.x);
  if (oar.world) {
    // publish the partial output: the last CTA to finish pushes Y (M x N, complete once every
    // CTA's writes are visible) into slot `rank` of every rank's mailbox with 16-byte stores,
    // fences them at system scope, bumps the epoch and releases the flags
    __threadfence();
    consumer_barrier<NC>();
    if (threadIdx.x == 0) flags[1] = atomicAdd(&oar.ctrs[1], 1u) == gridDim.x * gridDim.y - 1;
    consumer_barrier<NC>();
    if (flags[1]) {
      __threadfence();
      const size_t bytes = (size_t)M * N * sizeof(T);  // multiple of 16 (N % 8 == 0)
      const size_t off = kArFlagsBytes + (size_t)(oepoch & 1) * oar.region_bytes + (size_t)oar.rank * oar.slot_bytes;
      const uint4* src = reinterpret_cast<const uint4*>(Y);
      for (int d = 0; d < oar.world; ++d) {
        uint4* dst = reinterpret_cast<uint4*>(oar.mbox[d] + off);
        for (size_t i = threadIdx.x; i < bytes / 16; i += NC * 32) dst[i] = __ldcg(src + i);
      }
      __threadfence_system();
      consumer_barrier<NC>();
      if (threadIdx.x == 0) {
        oar.ctrs[1] = 0;
        oar.ctrs[0] = oepoch;
        for (int d = 0; d < oar.world; ++d)
          st_release_sys(reinterpret_cast<unsigned*>(oar.mbox[d]) + oar.rank, oepoch);
      }
    }
  }
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

}  // namespace

cudaError_t launch_mnb_prepack(const uint8_t* B, const void* scales, const uint8_t* zp, int scale_dtype,
                               const MnbPacked& p, cudaStream_t st) {
  if (scale_dtype == kF16) return prepack_b<__half>(B, scales, zp, p, st);
  if (scale_dtype == kBF16) return prepack_b<__nv_bfloat16>(B, scales, zp, p, st);
  return cudaErrorInvalidValue;
}

DeviceErrorSlot* device_error_slot();

namespace {
constexpr size_t kSmemCap = 232448;  // dynamic shared memory per CTA on sm_100

template <typename T, int BLOCK, int NT, bool PAIR, int G>
cudaError_t launch_tma_g(const void* A, const MnbPacked& p, void* Y, int64_t M, cudaStream_t st, const MnbPro& pro,
                         const MnbAr& oar, int xrows, int xmode, size_t x_bytes) {
  using RC = Rec<BLOCK>;
  // 16-token chunks stage 16 activation rows: one CTA per SM, so it gets twice the consumer warps
  constexpr int NC = NT == 2 ? 2 * kNC : kNC;
  constexpr int kMinC = NC > kNC ? 1 : kMinCtas;
  auto kern = mnb_tma_kernel<T, BLOCK, NT, PAIR, NC, G>;
  auto smem_for = [&](int stages) {
    const size_t stage = (size_t)G * RC::kBytes + (xmode == 2 ? (size_t)8 * NT * kXcStride : 0);
    return 256 + (size_t)stages * stage + (size_t)2 * NC * NT * 4 * 32 * 4 + (xrows ? x_bytes : 0);
  };
  static size_t configured = 0;        // per instantiation: the largest dynamic smem set so far
  auto configure = [&](size_t smem) -> cudaError_t {
    if (smem <= configured) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) configured = smem;
    return e;
  };
  // deepest ring that still leaves kMinCtas CTAs per SM (weights in flight per SM ~ kMinCtas x ring),
  // else the deepest ring that fits one CTA
  static size_t occ_key[8] = {};
  static int occ_val[8] = {};
  auto per_sm_for = [&](size_t smem, int* out) -> cudaError_t {
    for (int i = 0; i < 8; ++i)
      if (occ_key[i] == smem) return (*out = occ_val[i]), cudaSuccess;
    int n = 0;
    if (cudaError_t e = configure(smem)) return e;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, (NC + 1) * 32, smem);
    if (e != cudaSuccess) return e;
    for (int i = 0; i < 8; ++i)
      if (!occ_key[i]) {
        occ_key[i] = smem, occ_val[i] = n;
        break;
      }
    return (*out = n), cudaSuccess;
  };
  int stages = 0, per_sm = 0, fallback = 0, fallback_n = 0;
  for (int sg = kMaxStages; sg >= 2; --sg) {
    if (smem_for(sg) > kSmemCap) continue;
    int n = 0;
    if (cudaError_t e = per_sm_for(smem_for(sg), &n)) return e;
    if (n >= 1 && !fallback) fallback = sg, fallback_n = n;
    if (n >= kMinC) {
      stages = sg, per_sm = n;
      break;
    }
  }
  if (!stages) {
    if (!fallback) return cudaErrorInvalidValue;  // not even a 2-stage ring fits
    stages = fallback, per_sm = fallback_n;
  }
  if (cudaError_t e = configure(smem_for(stages))) return e;
  const size_t smem = smem_for(stages);
  const unsigned gy = (unsigned)((M + 8 * NT - 1) / (8 * NT));
  const int64_t ctas = std::min<int64_t>(p.ntiles, (int64_t)per_sm * num_sms());
  return launch_k(kern, dim3((unsigned)ctas, gy), dim3((NC + 1) * 32), smem, st, static_cast<const T*>(A),
                  static_cast<const uint8_t*>(p.w), static_cast<T*>(Y), (int)M, (int)p.N, (int)p.K, (int)p.ntiles,
                  (int)p.ksteps4, xrows, xmode, 0u, stages, pro, oar, device_error_slot());
}

template <typename T, int BLOCK, int NT, bool PAIR>
cudaError_t launch_tma_t(const void* A, const MnbPacked& p, void* Y, int64_t M, cudaStream_t st, const MnbPro& pro,
                         const MnbAr& oar) {
  // activation rows staged in shared memory when they fit (M = 1: K <= 16K)
  const int rows = (int)std::min<int64_t>(8 * NT, M);
  const size_t x_bytes = (size_t)(rows + 1) * (p.ksteps4 * 64 * 2 + 16);
  const bool a16 = (reinterpret_cast<uintptr_t>(A) & 15) == 0;  // staging reads 16-byte chunks
  const int xrows = x_bytes <= kXStageMax && (a16 || pro.kind != kProNone) ? rows : 0;
  if (pro.kind != kProNone && !xrows) return cudaErrorInvalidValue;  // caller checks mnb_prologue_fits
  // activation modes: 1 = all rows staged once per CTA; 2 = each stage's k-range bulk-copied beside
  // its records (rows too long to stage whole, e.g. 16 rows at K 14336); 0 = read from global memory
  const int xmode = xrows ? 1 : (a16 && p.K % 64 == 0 && p.ksteps4 * 64 == p.K) ? 2 : 0;
  // long streams of whole kGLong-record stages (at least three per CTA) run the long stages when a
  // two-stage ring of them, the merge buffers and the staged rows fit one CTA
  const int64_t per_cta = (int64_t)p.ntiles * p.ksteps4 / std::max<int64_t>(1, std::min<int64_t>(p.ntiles, 2 * num_sms()));
  constexpr int NCx = NT == 2 ? 2 * kNC : kNC;
  const size_t smem_long = 256 + (size_t)2 * kGLong * Rec<BLOCK>::kBytes + (size_t)2 * NCx * NT * 4 * 32 * 4 + x_bytes;
  if (xmode == 1 && p.ksteps4 % kGLong == 0 && per_cta >= 3 * kGLong && smem_long <= kSmemCap)
    return launch_tma_g<T, BLOCK, NT, PAIR, kGLong>(A, p, Y, M, st, pro, oar, xrows, xmode, x_bytes);
  return launch_tma_g<T, BLOCK, NT, PAIR, kG>(A, p, Y, M, st, pro, oar, xrows, xmode, x_bytes);
}

template <typename T, int BLOCK>
cudaError_t launch_nt(const void* A, const MnbPacked& p, void* Y, int64_t M, cudaStream_t st, const MnbPro& pro,
                      const MnbAr& oar) {
  if (M == 1) return launch_tma_t<T, BLOCK, 1, false>(A, p, Y, M, st, pro, oar);
  return M <= 8 ? launch_tma_t<T, BLOCK, 1, true>(A, p, Y, M, st, pro, oar)
                : launch_tma_t<T, BLOCK, 2, true>(A, p, Y, M, st, pro, oar);
}

template <typename T>
cudaError_t launch_b(const void* A, const MnbPacked& p, void* Y, int64_t M, cudaStream_t st, const MnbPro& pro,
                     const MnbAr& oar) {
  switch (p.block) {
    case 16: return launch_nt<T, 16>(A, p, Y, M, st, pro, oar);
    case 32: return launch_nt<T, 32>(A, p, Y, M, st, pro, oar);
    case 64: return launch_nt<T, 64>(A, p, Y, M, st, pro, oar);
    case 128: return launch_nt<T, 128>(A, p, Y, M, st, pro, oar);
  }
  return cudaErrorInvalidValue;
}
}  // namespace

cudaError_t launch_mnb_packed(const void* A, const MnbPacked& p, void* Y, int dtype, int64_t M, cudaStream_t st,
                              const MnbPro* pro, const MnbAr* out_ar) {
  if (M == 0) return cudaSuccess;
  const MnbPro none{};
  const MnbAr no_ar{};
  const MnbPro& pr = pro ? *pro : none;
  const MnbAr& oa = out_ar ? *out_ar : no_ar;
  if (dtype == kF16) return launch_b<__half>(A, p, Y, M, st, pr, oa);
  if (dtype == kBF16) return launch_b<__nv_bfloat16>(A, p, Y, M, st, pr, oa);
  return cudaErrorInvalidValue;
}

bool mnb_prologue_fits(int64_t M, int64_t K, int block) {
  const MnbPacked g = mnb_packed_geometry(1, K, block);
  const int64_t rows = std::min<int64_t>(M <= 8 ? 8 : 16, M);
  // every CTA of the GEMV recomputes the fused producer over all rows from L2, which pays for one
  // or two rows (measured on B200: batch 4 decodes faster with the standalone producer kernel and
  // plain staging); more than 16 rows run the tensor-core GEMM
  return M > 0 && M <= 2 && K % 8 == 0 && (size_t)M * K * 2 <= 32 * 1024 &&
         (size_t)(rows + 1) * (g.ksteps4 * 64 * 2 + 16) <= kXStageMax;
}

}  // namespace b200ep
