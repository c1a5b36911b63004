// Prompt attention (S > 1, head size 128, fp16 / bf16) on the 5th-generation tensor cores, after
// gqa_append_kernel has rotated the query rows into the fp32 workspace (rounded through T) and
// appended the rotated k and v rows (reference: the causal SDPA of the GroupQueryAttention handler,
// rust/src/ops/attention.rs:308-313 and 893-921, bottom-right-aligned causal mask with the optional
// local window).
//
// gqa_vt_kernel       copies each (batch, kv head)'s visible value rows transposed into a workspace
//                     V^T [B, HK, 128, LT] (zeros up to the next 128-key boundary), so that both
//                     products read K-major operands.
// gqa_umma_prefill_kernel — one CTA per (128 query rows, query head, batch), 18 warps:
//   warp 0 (one lane)  TMA: K tiles [128 keys x 128 d] from the KV buffer and V^T tiles [128 d x 128
//                      keys] from the workspace, both as two 64-element boxes with 128-byte swizzle,
//                      into two-stage rings;
//   warp 1 (one lane)  tcgen05.mma.kind::f16 (128 x 128 x 16, fp32 in TMEM): S_j = Q K_j^T into one
//                      of two S buffers, O += P_j V_j once P_j is in shared memory (two P buffers),
//                      then S_{j+2}; so the softmax of tile j + 1 overlaps P V of tile j;
//   warps 2..17        stage the query rows (fp32 workspace -> T, swizzled) once, then the softmax:
//                      warp w takes the rows of TMEM lane quarter w % 4 (one row per thread) and 32
//                      of the tile's 128 keys, (w - 2) / 4; per tile it reads its 32 scores
//                      (tcgen05.ld), the four warps of a quarter combine their row maxima through
//                      TMEM columns and a named barrier, then p = exp2(s - m) in fp32 (MUFU), summed
//                      unrounded per warp and stored rounded to T (packed conversions) as the A
//                      operand of P V; at the end the four partial sums are combined the same way
//                      and each warp writes its 32 columns of O / l.
// The reference maximum m of a row moves only when the row's maximum exceeds it by more than 8 (in
// log2 units); then O is rescaled in TMEM (tcgen05.ld / st) after the previous P V completes.  So
// p <= 256 and O is rarely touched.  Otherwise the arithmetic is that of gqa_mma_prefill_kernel
// (base-2 online softmax, P rounded to T for the product, fp32 accumulation, O / l at the end).
// Every mbarrier wait is bounded (timeout -> device error word).
#include <cuda.h>

#include <algorithm>
#include <cstdlib>

#include "../common.cuh"
#include "kernels.h"

namespace b200ep {

DeviceErrorSlot* device_error_slot();

namespace {

constexpr int kUR = 128;  // query rows per CTA
constexpr int kUK = 128;  // keys per tile
constexpr int kUD = 128;  // head size
constexpr int kUSoft = 16;                      // softmax warps: 4 per TMEM lane quarter, 32 keys each
constexpr int kUThreads = (2 + kUSoft) * 32;     // + the TMA and MMA warps
enum { kErrUmmaTimeout = 105 };

struct USmem {
  static constexpr int kBox = 128 * 128;      // 128 rows x 64 elements (128 B), 128-byte swizzle
  static constexpr int kQ = 0;                // [2 boxes]: d 0-63, 64-127
  static constexpr int kK = kQ + 2 * kBox;    // [2 stages][2 boxes] (rows = keys)
  static constexpr int kV = kK + 4 * kBox;    // [2 stages][2 boxes] (rows = d, 64 keys per box)
  static constexpr int kP = kV + 4 * kBox;    // [2 buffers][2 boxes]: keys 0-63, 64-127
  // kfull[2] kempty[2] vfull[2] vempty[2] sfull[2] pfull[2] pfree[2] odone qfull ofin fin
  static constexpr int kBar = kP + 4 * kBox;
  static constexpr int kNBar = 18;
  static constexpr int kTmemSlot = kBar + kNBar * 8;
  static constexpr int kTotal = kTmemSlot + 16 + 1024;  // + alignment slack
};
static_assert(USmem::kTotal <= 232448, "shared memory per CTA");

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_byte_addr) {
  // K-major, 128-byte swizzle: 8-row groups 1024 bytes apart (SBO), LBO unused (1), version 1
  uint64_t d = 0;
  d |= (uint64_t)((smem_byte_addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

template <typename T>
__device__ __forceinline__ uint32_t idesc_128x128() {
  constexpr uint32_t fmt = std::is_same<T, __half>::value ? 0u : 1u;  // A / B type; D = fp32
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(128 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(tmem_d),
      "l"(ad), "l"(bd), "r"(idesc), "r"(acc), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 32 consecutive columns of this thread's lane; tmem_wait_ld() before the values are used
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// byte offset of element (row, k) in a 128-row x 64-element K-major box with 128-byte swizzle
__device__ __forceinline__ uint32_t sw128_off(int row, int k) {
  return (uint32_t)(row * 128 + ((((k >> 3) ^ (row & 7)) & 7) << 4) + (k & 7) * 2);
}

// two values rounded to T in one packed conversion (a in the low half)
template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float a, float b) {
  if constexpr (std::is_same<T, __half>::value) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

// 2^x by the hardware approximation (MUFU.EX2; subnormal results flush to zero)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// warp-uniform bounded wait
__device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t phase) {
  return __all_sync(0xffffffffu, mbar_wait(bar, phase));
}

__device__ __forceinline__ int umma_past(const UmmaAttnArgs& a, int b) { return a.seqlens[b] + 1 - a.S; }
__device__ __forceinline__ bool umma_ok(const UmmaAttnArgs& a, int past) {
  return past >= 0 && past + a.S <= a.cap && (!a.do_rotary || past + a.S <= a.max_seq);
}

template <typename T>
__global__ void __launch_bounds__(256) gqa_vt_kernel(UmmaAttnArgs a) {
  pdl_wait();  // the append kernel wrote this prompt's v rows
  pdl_trigger();
  const int b = blockIdx.z, kvh = blockIdx.y, key0 = blockIdx.x * 64;
  const int past = umma_past(a, b);
  const int L = umma_ok(a, past) ? past + a.S : 0;
  if (key0 >= (L + kUK - 1) / kUK * kUK) return;
  __shared__ __align__(16) T tile[64][kUD + 8];
  const T* src = static_cast<const T*>(a.kv_v) + ((int64_t)(b * a.HK + kvh) * a.cap + key0) * kUD;
  for (int i = threadIdx.x; i < 64 * (kUD / 8); i += blockDim.x) {
    const int kr = i / (kUD / 8), ch = i % (kUD / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (key0 + kr < L) v = *reinterpret_cast<const uint4*>(src + (int64_t)kr * kUD + ch * 8);
    *reinterpret_cast<uint4*>(&tile[kr][ch * 8]) = v;
  }
  __syncthreads();
  T* dst = static_cast<T*>(a.vt) + (int64_t)(b * a.HK + kvh) * kUD * a.lt + key0;
  for (int i = threadIdx.x; i < kUD * 8; i += blockDim.x) {
    const int d = i / 8, kc = i % 8;
    uint4 pk;
    T* h = reinterpret_cast<T*>(&pk);
#pragma unroll
    for (int u = 0; u < 8; ++u) h[u] = tile[kc * 8 + u][d];
    *reinterpret_cast<uint4*>(dst + (int64_t)d * a.lt + kc * 8) = pk;
  }
}

template <typename T>
__global__ void __launch_bounds__(kUThreads, 1)
gqa_umma_prefill_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                        UmmaAttnArgs a) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + USmem::kBar);
  uint64_t* kfull = bars;
  uint64_t* kempty = bars + 2;
  uint64_t* vfull = bars + 4;
  uint64_t* vempty = bars + 6;
  uint64_t* sfull = bars + 8;
  uint64_t* pfull = bars + 10;
  uint64_t* pfree = bars + 12;
  uint64_t* odone = bars + 14;
  uint64_t* qfull = bars + 15;
  uint64_t* ofin = bars + 16;
  uint64_t* fin = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + USmem::kTmemSlot);
  int* flag = reinterpret_cast<int*>(sm + USmem::kTmemSlot + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int xb = (int)gridDim.x - 1 - (int)blockIdx.x;  // the longest causal rows start first
  const int h = blockIdx.y, b = blockIdx.z, kvh = h / a.G;
  const int S = a.S;
  const int past = umma_past(a, b);
  const int i0 = xb * kUR;
  if (!umma_ok(a, past) || i0 >= S) return;  // reported by gqa_append_kernel; uniform for the CTA
  const int ilast = min(S, i0 + kUR) - 1;
  const int win = a.local_window;
  const int lo_blk = win > 0 ? max(0, past + i0 - win + 1) : 0;
  const int hi_blk = past + ilast;
  const int t0 = lo_blk / kUK, nt = hi_blk / kUK - t0 + 1;
  const int krow0 = (b * a.HK + kvh) * a.cap;  // K map row of key 0
  const int vrow0 = (b * a.HK + kvh) * kUD;    // V^T map row of dimension 0

  if (threadIdx.x == 0) {
    *flag = 0;
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kfull[s], 1);
      mbar_init(&kempty[s], 1);
      mbar_init(&vfull[s], 1);
      mbar_init(&vempty[s], 1);
      mbar_init(&sfull[s], 1);
      mbar_init(&pfull[s], kUSoft);
      mbar_init(&pfree[s], 1);
    }
    mbar_init(odone, 1);
    mbar_init(qfull, kUSoft);
    mbar_init(ofin, 1);
    mbar_init(fin, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;  // S buffers at columns 0 and 128, O at 256
  pdl_wait();  // q rows, k / v rows and V^T are the previous kernels' output
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      for (int j = 0; j < nt; ++j) {
        const int s = j & 1, key0 = (t0 + j) * kUK;
        if (j >= 2 && !mbar_wait(&kempty[s], ((j >> 1) - 1) & 1)) {
          *flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&kfull[s], 2 * USmem::kBox);
        tma_2d(sm + USmem::kK + (s * 2) * USmem::kBox, &kmap, 0, krow0 + key0, &kfull[s]);
        tma_2d(sm + USmem::kK + (s * 2 + 1) * USmem::kBox, &kmap, 64, krow0 + key0, &kfull[s]);
        if (j >= 2 && !mbar_wait(&vempty[s], ((j >> 1) - 1) & 1)) {
          *flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&vfull[s], 2 * USmem::kBox);
        tma_2d(sm + USmem::kV + (s * 2) * USmem::kBox, &vmap, key0, vrow0, &vfull[s]);
        tma_2d(sm + USmem::kV + (s * 2 + 1) * USmem::kBox, &vmap, key0 + 64, vrow0, &vfull[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_128x128<T>();
      const uint32_t qa = smem_u32(sm + USmem::kQ), ka = smem_u32(sm + USmem::kK);
      const uint32_t va = smem_u32(sm + USmem::kV), pa = smem_u32(sm + USmem::kP);
      bool alive = mbar_wait(qfull, 0);
      auto issue_s = [&](int j) {
        const int s = j & 1;
        if (!mbar_wait(&kfull[s], (j >> 1) & 1)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
        for (int kk = 0; kk < kUD / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * USmem::kBox + (kk & 3) * 32);
          umma_f16(tmem + (uint32_t)(s * 128), umma_desc_sw128(qa + off),
                   umma_desc_sw128(ka + (uint32_t)(s * 2 * USmem::kBox) + off), idesc, kk > 0 ? 1u : 0u);
        }
        umma_commit(&kempty[s]);
        umma_commit(&sfull[s]);
        return true;
      };
      if (alive) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        alive = issue_s(0) && (nt < 2 || issue_s(1));
      }
      // P V of tile j once its P is written; then S of tile j + 2 into the S buffer tile j used
      // (its softmax has read it: P_j is written after).  The softmax of tile j + 1 runs meanwhile.
      for (int j = 0; j < nt && alive; ++j) {
        if (!mbar_wait(&pfull[j & 1], (j >> 1) & 1) || !mbar_wait(&vfull[j & 1], (j >> 1) & 1)) {
          alive = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
        for (int kk = 0; kk < kUK / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * USmem::kBox + (kk & 3) * 32);
          umma_f16(tmem + 256u, umma_desc_sw128(pa + (uint32_t)((j & 1) * 2 * USmem::kBox) + off),
                   umma_desc_sw128(va + (uint32_t)((j & 1) * 2 * USmem::kBox) + off), idesc,
                   (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&vempty[j & 1]);
        umma_commit(&pfree[j & 1]);
        umma_commit(odone);
        if (j + 2 < nt && !(alive = issue_s(j + 2))) break;
      }
      umma_commit(ofin);
      if (!alive) *flag = 1;
      // every MMA of this CTA has completed before the tensor memory is released
      umma_commit(fin);
      if (!mbar_wait(fin, 0)) *flag = 1;
    }
    __syncwarp();
  } else {
    // warps 2..17: the 128 query rows (fp32 workspace, already rounded through T) into the two
    // swizzled Q boxes
    {
      const int t = (int)threadIdx.x - 64;
      for (int it = t; it < kUR * (kUD / 8); it += kUSoft * 32) {
        const int row = it / (kUD / 8), ch = it % (kUD / 8);
        const int i = i0 + row;
        float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (i < S) {
          const float4* src = reinterpret_cast<const float4*>(a.qrot + (((int64_t)b * S + i) * a.H + h) * kUD + ch * 8);
          const float4 x0 = src[0], x1 = src[1];
          f[0] = x0.x, f[1] = x0.y, f[2] = x0.z, f[3] = x0.w, f[4] = x1.x, f[5] = x1.y, f[6] = x1.z, f[7] = x1.w;
        }
        const uint4 pk = make_uint4(pack_pair<T>(f[0], f[1]), pack_pair<T>(f[2], f[3]), pack_pair<T>(f[4], f[5]),
                                    pack_pair<T>(f[6], f[7]));
        *reinterpret_cast<uint4*>(sm + USmem::kQ + (ch >> 3) * USmem::kBox + sw128_off(row, (ch & 7) * 8)) = pk;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(qfull);
    }
    // softmax: warp w owns TMEM lane quarter q = w % 4 (rows 32 q .. 32 q + 31, one per thread) and
    // key / output column chunk c = (w - 2) / 4 (32 of the tile's 128 keys, 32 of O's 128 columns).
    // The four warps of a quarter combine their row maxima through TMEM columns 384.. (named
    // barrier 1 + q), so every one of them holds the same reference maximum per row.
    {
      const int q = warp & 3, c = (warp - 2) >> 2;
      const int r = q * 32 + lane;
      const int i = i0 + r;
      const bool valid = i < S;
      const int pos = past + i;
      const int lo = win > 0 ? max(0, pos - win + 1) : 0;
      const uint32_t lbase = tmem + ((uint32_t)(q * 32) << 16);
      auto group_sync = [&]() {
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        asm volatile("bar.sync %0, 128;" ::"r"(1 + q) : "memory");
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      };
      // this warp's value in TMEM column `col` (one per row) and the four warps' values back
      auto exchange4 = [&](uint32_t col, float x, float (&all)[4]) {
        uint32_t xv = __float_as_uint(x);
        asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(lbase + col + (uint32_t)c), "r"(xv)
                     : "memory");
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        group_sync();
        uint32_t u0, u1, u2, u3;
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(u0), "=r"(u1), "=r"(u2), "=r"(u3)
                     : "r"(lbase + col));
        tmem_wait_ld();
        all[0] = __uint_as_float(u0), all[1] = __uint_as_float(u1), all[2] = __uint_as_float(u2);
        all[3] = __uint_as_float(u3);
      };
      // Every warp of a quarter runs every iteration and both exchanges (its named barrier must
      // see all four), so a timed-out wait only marks the warp dead: it stops waiting and its
      // results are discarded.
      float m_ref = -INFINITY, l = 0.f;
      bool alive = true;
      for (int j = 0; j < nt; ++j) {
        const int s = j & 1, key0 = (t0 + j) * kUK + c * 32;
        alive = alive && wait_all(&sfull[s], (j >> 1) & 1);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        // this warp's 32 keys of the row of S_j, scaled to the base-2 exponent domain
        uint32_t v[32];
        tmem_ld32(lbase + (uint32_t)(s * 128 + c * 32), v);
        // every key of the warp's 32 x 32 block visible (all but the diagonal and window edges):
        // raw scores, scaled inside the exponent; otherwise scaled scores with -inf where masked
        const bool wfull = __all_sync(0xffffffffu, valid && key0 >= lo && key0 + 31 <= pos && a.scale_log2 > 0.f);
        float mxs[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (wfull) {
#pragma unroll
          for (int e = 0; e < 32; ++e) mxs[e & 3] = fmaxf(mxs[e & 3], __uint_as_float(v[e]));
#pragma unroll
          for (int u = 0; u < 4; ++u) mxs[u] *= a.scale_log2;
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int key = key0 + e;
            const float x = __uint_as_float(v[e]) * a.scale_log2;
            const bool vis = valid && key >= lo && key <= pos;
            v[e] = __float_as_uint(vis ? x : -INFINITY);
            mxs[e & 3] = fmaxf(mxs[e & 3], vis ? x : -INFINITY);
          }
        }
        float part[4];
        exchange4(384u + (uint32_t)((j & 1) * 4), fmaxf(fmaxf(mxs[0], mxs[1]), fmaxf(mxs[2], mxs[3])), part);
        const float mx = fmaxf(fmaxf(part[0], part[1]), fmaxf(part[2], part[3]));
        // P buffer j & 1 belongs to P V of tile j - 2 until it completes
        if (j >= 2) alive = alive && wait_all(&pfree[j & 1], ((j >> 1) - 1) & 1);
        // the reference maximum moves only when the row's maximum exceeds it by more than 2^8, so
        // p = exp2(s - m_ref) <= 256 and O is rescaled rarely
        const bool grow = mx > m_ref + 8.f || (m_ref == -INFINITY && mx != -INFINITY);
        const float alpha = grow ? (m_ref == -INFINITY ? 0.f : exp2f(m_ref - mx)) : 1.f;
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
          // O holds every earlier tile's P V once tile j - 1's completes (tile j's is not issued)
          alive = alive && wait_all(odone, (j - 1) & 1);
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          uint32_t o[32];
          tmem_ld32(lbase + 256u + (uint32_t)(c * 32), o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(lbase + 256u + (uint32_t)(c * 32), o);
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        l *= alpha;
        if (grow) m_ref = mx;
        // a row without a visible key so far has only -inf scores: any finite reference gives 0
        const float mr = m_ref == -INFINITY ? 0.f : m_ref;
        float pss[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t pk[16];
        if (wfull) {
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float x0 = fmaf(__uint_as_float(v[e]), a.scale_log2, -mr);
            const float x1 = fmaf(__uint_as_float(v[e + 1]), a.scale_log2, -mr);
            const float p0 = ex2(x0);
            const float p1 = ex2(x1);
            pss[(e >> 1) & 3] += p0 + p1;
            pk[e >> 1] = pack_pair<T>(p0, p1);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float p0 = ex2(__uint_as_float(v[e]) - mr);  // -inf (masked) -> 0
            const float p1 = ex2(__uint_as_float(v[e + 1]) - mr);
            pss[(e >> 1) & 3] += p0 + p1;
            pk[e >> 1] = pack_pair<T>(p0, p1);
          }
        }
        const uint32_t pb = smem_u32(sm + USmem::kP + ((j & 1) * 2 + (c >> 1)) * USmem::kBox);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          sts128(pb + sw128_off(r, (c & 1) * 32 + u * 8), make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]));
        l += (pss[0] + pss[1]) + (pss[2] + pss[3]);  // this warp's keys; summed across warps at the end
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&pfull[j & 1]);
      }
      // every warp of the quarter takes part in the final exchange, also after a timeout
      if (!alive) l = 0.f;
      const bool done = alive && wait_all(ofin, 0);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      float part[4];
      exchange4(392u, l, part);
      const float lt = (part[0] + part[1]) + (part[2] + part[3]);
      if (done) {
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
        uint32_t o[32];
        tmem_ld32(lbase + 256u + (uint32_t)(c * 32), o);
        if (valid) {
          T* orow = static_cast<T*>(a.out) + (((int64_t)b * S + i) * a.H + h) * kUD + c * 32;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint4 pk = make_uint4(pack_pair<T>(__uint_as_float(o[8 * u]) * inv, __uint_as_float(o[8 * u + 1]) * inv),
                                        pack_pair<T>(__uint_as_float(o[8 * u + 2]) * inv, __uint_as_float(o[8 * u + 3]) * inv),
                                        pack_pair<T>(__uint_as_float(o[8 * u + 4]) * inv, __uint_as_float(o[8 * u + 5]) * inv),
                                        pack_pair<T>(__uint_as_float(o[8 * u + 6]) * inv, __uint_as_float(o[8 * u + 7]) * inv));
            *reinterpret_cast<uint4*>(orow + u * 8) = pk;
          }
        }
      }
      if (!done && lane == 0) *flag = 1;
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
  if (*flag && threadIdx.x == 0) report_device_error(a.err, kErrUmmaTimeout, b);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D map over rows of `inner` 16-bit elements, boxes of 64 elements x 128 rows, 128-byte swizzle
bool make_map(CUtensorMap* map, int dtype, const void* base, uint64_t inner, uint64_t rows) {
  EncodeTiledFn enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
  const cuuint32_t box[2] = {64, 128};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  return enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T>
cudaError_t launch_umma_t(const UmmaAttnArgs& a, cudaStream_t st) {
  CUtensorMap kmap, vmap;
  if (!make_map(&kmap, a.dtype, a.kv_k, kUD, (uint64_t)a.B * a.HK * a.cap) ||
      !make_map(&vmap, a.dtype, a.vt, (uint64_t)a.lt, (uint64_t)a.B * a.HK * kUD))
    return cudaErrorInvalidValue;
  cudaError_t e = launch_k(gqa_vt_kernel<T>, dim3((unsigned)(a.lt / 64), (unsigned)a.HK, (unsigned)a.B), dim3(256), 0,
                           st, a);
  if (e != cudaSuccess) return e;
  auto kern = gqa_umma_prefill_kernel<T>;
  static bool configured = false;
  if (!configured) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, USmem::kTotal);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return launch_k(kern, dim3((unsigned)((a.S + kUR - 1) / kUR), (unsigned)a.H, (unsigned)a.B), dim3(kUThreads),
                  (size_t)USmem::kTotal, st, kmap, vmap, a);
}

}  // namespace

int64_t gqa_umma_lt(int64_t cap) { return (cap + kUK - 1) / kUK * kUK; }

size_t gqa_umma_vt_bytes(int64_t batch, int64_t kv_heads, int64_t cap) {
  return (size_t)batch * kv_heads * kUD * gqa_umma_lt(cap) * 2;
}

bool gqa_umma_supported(int64_t batch, int64_t kv_heads, int64_t head_size, int64_t cap, int dtype) {
  static const bool off = std::getenv("ONNXRUNTIME_EP_B200_NO_UMMA_ATTN") != nullptr;
  // TMA row coordinates are 32-bit
  return !off && head_size == kUD && (dtype == kF16 || dtype == kBF16) &&
         batch * kv_heads * gqa_umma_lt(cap) < ((int64_t)1 << 31);
}

cudaError_t launch_gqa_umma_prefill(const UmmaAttnArgs& a, cudaStream_t st) {
  return a.dtype == kF16 ? launch_umma_t<__half>(a, st) : launch_umma_t<__nv_bfloat16>(a, st);
}

}  // namespace b200ep
