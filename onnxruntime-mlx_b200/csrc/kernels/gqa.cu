// GroupQueryAttention for sm_100a (reference: group_query_attention_op,
// rust/src/ops/attention.rs:556-952, which composes mlx_fast_rope, mlx_slice_update and
// mlx_fast_scaled_dot_product_attention).
//
// gqa_decode_kernel — split-K flash-decode over the shared KV buffer.
//   grid (splits, kv_heads, batch); 4 consumer warps + 1 producer warp.
//   * Every CTA rotates (RoPE, optional per-head RMS norm) the R = S * (H / HK) query rows of its
//     kv-head group into shared memory, rounded through the I/O dtype as ORT stores them.
//   * The CTA whose key range holds the new positions [past_b, past_b + S) rotates the new k rows
//     and writes k and v in place into the KV buffer (the fused KV append), then fences the
//     generic-proxy writes against the TMA reads that follow.
//   * The producer warp streams 32-key K/V tiles with 1-D bulk copies (cp.async.bulk, the TMA
//     engine) into a ring of shared-memory stages guarded by mbarriers; all waits are bounded.
//   * Consumers: each lane owns head_size/32 contiguous dims of a key; q.k partials for
//     (keys x rows) are reduce-scattered across the warp so each lane ends with one score, then
//     an fp32 online softmax (base 2) and the P.V accumulation run per warp.
//   * Warp states merge in shared memory; with splits > 1 each CTA writes (m, l, o) partials and
//     the last CTA of its (batch, kv-head) — found with an arrival counter that it resets —
//     merges them into the output.
// past_b = seqlens_k[b] + 1 - S is read on the device, so a launch configuration (and a CUDA
// graph holding it) serves every decode step.
//
// gqa_append_kernel + gqa_mma_prefill_kernel — prompt rows (S > 1, fp16 / bf16, head_size 64 or
// 128): the append kernel rotates and appends, a tensor-core flash-attention kernel attends.
//
// gqa_append_kernel + gqa_generic_kernel — the same semantics for shapes the other kernels
// do not cover (head_size not a multiple of 32, more than 32 query rows per group, unaligned
// rows): one CTA per query row, keys in shared memory.
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "../common.cuh"
#include "kernels.h"

namespace b200ep {

DeviceErrorSlot* device_error_slot();

enum GqaErr { kErrGqaRange = 101, kErrGqaTimeout = 102 };

struct GqaKP {
  const void* q;
  const void* k;
  const void* v;
  void* kv_k;
  void* kv_v;
  const int32_t* seqlens;
  const void* cos_c;
  const void* sin_c;
  const void* qn;
  const void* kn;
  const void* bias;
  void* out;
  float* partial;
  int* counters;
  float* qrot;  // generic path only
  DeviceErrorSlot* err;
  int B, S, H, HK, D, G, R, cap, max_seq, half, splits;
  int do_rotary, interleaved, local_window;
  int64_t qstride, kstride, koff, voff;  // element strides of the new-row inputs
  int bias_batch, bias_total;
  float scale_log2;  // scale * log2(e)
  float qk_eps;
  int has_qk_norm;
  // PagedAttention through gqa_mma_decode_kernel<..., true>: blockIdx.z is a packed row of
  // p_batch sequences (cumulative lengths p_cum, past lengths p_past); key j of its sequence lives
  // at cache row p_bt[seq][j / p_bs] * p_bs + j % p_bs of kv_k / kv_v [p_nblocks, p_bs, HK, D]
  const int32_t* p_cum;
  const int32_t* p_past;
  const int32_t* p_bt;
  int p_batch, p_nblocks, p_bs, p_maxb;
};

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kNW = 8;        // consumer warps
constexpr int kKT = 32;       // keys per stage
constexpr int kKPW = kKT / kNW;  // keys per warp per stage

// ---- shared prologue pieces -----------------------------------------------------------------
// Rotates (and optionally RMS-normalises) one head row held in `row` (fp32, D values) in place.
// Executed by one warp; `row` lives in shared memory.
template <typename T>
__device__ void rotate_row_warp(float* row, int D, int pos, const GqaKP& kp, const void* normw) {
  const int lane = threadIdx.x & 31;
  if (kp.has_qk_norm) {
    float ss = 0.f;
    for (int i = lane; i < D; i += 32) ss = fmaf(row[i], row[i], ss);
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / (float)D + kp.qk_eps);
    const T* w = static_cast<const T*>(normw);
    for (int i = lane; i < D; i += 32) row[i] = row[i] * inv * to_f<T>(w[i]);
    __syncwarp();
  }
  if (kp.do_rotary) {
    const T* cc = static_cast<const T*>(kp.cos_c) + (int64_t)pos * kp.half;
    const T* sc = static_cast<const T*>(kp.sin_c) + (int64_t)pos * kp.half;
    float o0[4], o1[4];  // rotary_half <= 128 -> at most 4 pairs per lane
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int i = lane + 32 * c;
      if (i < kp.half) {
        const float cs = to_f<T>(cc[i]), sn = to_f<T>(sc[i]);
        const int i0 = kp.interleaved ? 2 * i : i;
        const int i1 = kp.interleaved ? 2 * i + 1 : i + kp.half;
        const float a = row[i0], b = row[i1];
        o0[c] = a * cs - b * sn;
        o1[c] = b * cs + a * sn;
      }
    }
    __syncwarp();
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int i = lane + 32 * c;
      if (i < kp.half) {
        row[kp.interleaved ? 2 * i : i] = o0[c];
        row[kp.interleaved ? 2 * i + 1 : i + kp.half] = o1[c];
      }
    }
    __syncwarp();
  }
  for (int i = lane; i < D; i += 32) row[i] = round_through<T>(row[i]);
  __syncwarp();
}

__device__ __forceinline__ int past_len(const GqaKP& kp, int b) { return kp.seqlens[b] + 1 - kp.S; }

__device__ __forceinline__ bool range_ok(const GqaKP& kp, int past) {
  return past >= 0 && past + kp.S <= kp.cap && (!kp.do_rotary || past + kp.S <= kp.max_seq);
}

// ---- decode kernel --------------------------------------------------------------------------
struct DecodeSmem {
  // byte offsets inside dynamic shared memory
  int bars, kbuf, vbuf, qs, pbuf, wst, scratch, flags, total;
  int stages;
};

__host__ __device__ inline DecodeSmem decode_smem_layout(int D, int esz, int RP, int stages) {
  DecodeSmem L;
  L.stages = stages;
  int off = 0;
  L.bars = off;
  off += 2 * stages * 8;
  off = (off + 127) & ~127;
  const int tile = kKT * D * esz;
  L.kbuf = off;
  off += stages * tile;
  L.vbuf = off;
  off += stages * tile;
  L.qs = off;
  off += RP * D * 4;
  L.pbuf = off;
  off += kNW * 32 * 4;
  L.wst = off;
  off += kNW * RP * (D + 2) * 4;
  L.scratch = off;
  off += kNW * D * 4;
  L.flags = off;
  off += 16;
  L.total = off;
  return L;
}

__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Signal a named barrier without waiting for it to complete.
__device__ __forceinline__ void named_barrier_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

template <typename T, int EPL, int RP>
__global__ void __launch_bounds__((kNW + 1) * 32)
gqa_decode_kernel(GqaKP kp, int stages) {
  constexpr int D = EPL * 32;
  constexpr int KWW = (32 / RP) < kKPW ? (32 / RP) : kKPW;  // keys per warp step
  constexpr int NV = KWW * RP;                                // values per lane before the reduce
  static_assert(NV <= 32 && (NV & (NV - 1)) == 0, "NV must be a power of two <= 32");
  constexpr int LOGNV = NV == 1 ? 0 : NV == 2 ? 1 : NV == 4 ? 2 : NV == 8 ? 3 : NV == 16 ? 4 : 5;
  constexpr int SHIFT = 5 - LOGNV;
  constexpr bool QREG = RP * EPL <= 32;
  constexpr int kThreads = (kNW + 1) * 32;

  extern __shared__ __align__(128) unsigned char smem[];
  const DecodeSmem L = decode_smem_layout(D, (int)sizeof(T), RP, stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + stages;
  T* kbuf = reinterpret_cast<T*>(smem + L.kbuf);
  T* vbuf = reinterpret_cast<T*>(smem + L.vbuf);
  float* qs = reinterpret_cast<float*>(smem + L.qs);
  float* pbuf = reinterpret_cast<float*>(smem + L.pbuf);
  float* wst = reinterpret_cast<float*>(smem + L.wst);
  float* scratch = reinterpret_cast<float*>(smem + L.scratch);
  int* flags = reinterpret_cast<int*>(smem + L.flags);

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();  // the KV buffers and this step's q/k/v come from earlier kernels
  pdl_trigger();
  const int past = past_len(kp, b);
  const int total = past + kp.S;
  const bool ok = range_ok(kp, past);
  const int64_t head_base = ((int64_t)b * kp.HK + kvh) * kp.cap;  // row index of key 0
  T* kvk = static_cast<T*>(kp.kv_k) + head_base * D;
  T* kvv = static_cast<T*>(kp.kv_v) + head_base * D;

  // key range of this split
  int lo = 0;
  if (kp.local_window > 0) lo = max(0, past - kp.local_window + 1);
  const int span = max(total - lo, 0);
  int chunk = (span + kp.splits - 1) / kp.splits;
  chunk = ((chunk + kKT - 1) / kKT) * kKT;
  const int kbeg = ok ? min(lo + split * chunk, total) : 0;
  const int kend = ok ? min(kbeg + chunk, total) : 0;
  const int ntiles = (kend - kbeg + kKT - 1) / kKT;
  // this CTA appends new rows iff its range holds some of [past, total)
  const bool has_new = ok && kend > past && kbeg < total;

  if (threadIdx.x == 0) {
    flags[0] = 0;       // error flag
    flags[2] = 0;       // tiles issued by the producer
    flags[3] = ntiles;  // tiles every consumer warp finished (min)
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kNW);
    }
    fence_mbarrier_init();
    if (!ok && split == 0 && kvh == 0) report_device_error(kp.err, kErrGqaRange, b);
  }
  for (int i = threadIdx.x; i < (RP - kp.R) * D; i += kThreads) qs[kp.R * D + i] = 0.f;
  __syncthreads();

  if (warp == kNW) {
    // --- producer warp: stream K/V tiles from the start; the tile holding the new rows waits
    // for the consumers' append (named barrier 1).
    bool gated = false, alive = ok;
    for (int t = 0; t < ntiles && alive; ++t) {
      const int s = t % stages;
      const int j0 = kbeg + t * kKT;
      const int nk = min(kKT, kend - j0);
      if (has_new && !gated && j0 + nk > past) {
        named_barrier(1, kThreads);
        gated = true;
      }
      int go = 1;
      if (lane == 0) {
        if (t >= stages && !mbar_wait(&empty[s], ((t / stages) - 1) & 1)) {
          atomicExch(&flags[0], 1);
          go = 0;
        } else {
          const uint32_t bytes = (uint32_t)(nk * D * sizeof(T));
          mbar_arrive_expect_tx(&full[s], 2 * bytes);
          bulk_g2s(kbuf + (size_t)s * kKT * D, kvk + (int64_t)j0 * D, bytes, &full[s]);
          bulk_g2s(vbuf + (size_t)s * kKT * D, kvv + (int64_t)j0 * D, bytes, &full[s]);
          flags[2] = t + 1;
        }
      }
      alive = __shfl_sync(0xffffffffu, go, 0) != 0;
    }
    if (has_new && !gated) named_barrier(1, kThreads);
  } else {
    // --- consumer warps: prologue (rotated q rows; fused append of the new k / v rows) ------
    if (ok) {
      const T* qin = static_cast<const T*>(kp.q);
      for (int r = warp; r < kp.R; r += kNW) {
        const int s = r / kp.G, g = r - s * kp.G, h = kvh * kp.G + g;
        float* row = qs + r * D;
        const T* src = qin + ((int64_t)b * kp.S + s) * kp.qstride + (int64_t)h * D;
        for (int i = lane; i < D; i += 32) row[i] = to_f<T>(src[i]);
        __syncwarp();
        rotate_row_warp<T>(row, D, past + s, kp, kp.qn);
      }
      if (has_new) {
        const T* kin = static_cast<const T*>(kp.k);
        const T* vin = static_cast<const T*>(kp.v);
        for (int s = warp; s < kp.S; s += kNW) {
          const int pos = past + s;
          if (pos < kbeg || pos >= kend) continue;  // another split owns this row
          float* row = scratch + warp * D;
          const int64_t in_off = ((int64_t)b * kp.S + s) * kp.kstride + (int64_t)kvh * D;
          for (int i = lane; i < D; i += 32) row[i] = to_f<T>(kin[in_off + kp.koff + i]);
          __syncwarp();
          rotate_row_warp<T>(row, D, pos, kp, kp.kn);
          for (int i = lane; i < D; i += 32) {
            kvk[(int64_t)pos * D + i] = from_f<T>(row[i]);
            kvv[(int64_t)pos * D + i] = vin[in_off + kp.voff + i];
          }
        }
        fence_proxy_async_global();
        // release the producer's gated tile; never wait here (the producer may be blocked on a
        // free stage that only these warps can release)
        named_barrier_arrive(1, kThreads);
      }
    }
    named_barrier(2, kNW * 32);  // all q rows rotated

    float qreg[QREG ? RP : 1][EPL];
    if (QREG) {
#pragma unroll
      for (int r = 0; r < (QREG ? RP : 1); ++r)
#pragma unroll
        for (int e = 0; e < EPL; ++e) qreg[r][e] = qs[r * D + lane * EPL + e];
    }
    float m_run[RP], l_run[RP], o[RP][EPL];
#pragma unroll
    for (int r = 0; r < RP; ++r) {
      m_run[r] = -INFINITY;
      l_run[r] = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) o[r][e] = 0.f;
    }
    const int my_idx = lane >> SHIFT;  // value index this lane holds after the reduce-scatter
    const int my_r = my_idx % RP;
    const int my_kk = my_idx / RP;
    const int my_s = my_r / kp.G;
    const int qpos = past + my_s;
    const T* bias = static_cast<const T*>(kp.bias);
    const int64_t bias_row =
        kp.bias_batch > 0 ? ((int64_t)(kp.bias_batch == 1 ? 0 : b) * kp.S + my_s) * kp.bias_total : 0;

    for (int t = 0; t < ntiles; ++t) {
      const int s = t % stages;
      if (!mbar_wait(&full[s], (t / stages) & 1)) {
        atomicExch(&flags[0], 1);
        if (lane == 0) atomicMin(&flags[3], t);
        break;
      }
      const int j0 = kbeg + t * kKT;
      const T* kt = kbuf + (size_t)s * kKT * D;
      const T* vt = vbuf + (size_t)s * kKT * D;
#pragma unroll
      for (int step = 0; step < kKPW / KWW; ++step) {
        const int kl0 = warp * kKPW + step * KWW;  // first key (tile-local) of this step
        float v[NV];
#pragma unroll
        for (int kk = 0; kk < KWW; ++kk) {
          const int kl = kl0 + kk;
          float kf[EPL];
          const T* kr = kt + (size_t)kl * D + lane * EPL;
#pragma unroll
          for (int e = 0; e < EPL; ++e) kf[e] = (j0 + kl < kend) ? to_f<T>(kr[e]) : 0.f;
#pragma unroll
          for (int r = 0; r < RP; ++r) {
            float acc = 0.f;
#pragma unroll
            for (int e = 0; e < EPL; ++e) {
              const float qv = QREG ? qreg[QREG ? r : 0][e] : qs[r * D + lane * EPL + e];
              acc = fmaf(qv, kf[e], acc);
            }
            v[kk * RP + r] = acc;
          }
        }
        // reduce-scatter: lane ends with the full dot product of value index (lane >> SHIFT)
        int cur = NV;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
          if (cur > 1) {
            const int halfn = cur >> 1;
            const bool upper = (lane & off) != 0;
#pragma unroll
            for (int i = 0; i < NV / 2; ++i) {
              if (i < halfn) {
                const float send = upper ? v[i] : v[i + halfn];
                const float keep = upper ? v[i + halfn] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
              }
            }
            cur = halfn;
          } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
          }
        }
        const int j = j0 + kl0 + my_kk;
        float sc = v[0] * kp.scale_log2;
        const bool valid = (j < kend) && (my_r < kp.R) && (j <= qpos) &&
                           (kp.local_window <= 0 || j > qpos - kp.local_window);
        if (valid && bias && j < kp.bias_total) sc += to_f<T>(bias[bias_row + j]) * kLog2e;
        if (!valid) sc = -INFINITY;
        float mx = sc;
#pragma unroll
        for (int off = RP << SHIFT; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        float m_new[RP];
#pragma unroll
        for (int r = 0; r < RP; ++r) m_new[r] = fmaxf(m_run[r], __shfl_sync(0xffffffffu, mx, r << SHIFT));
        float mrow = m_new[0];
#pragma unroll
        for (int r = 1; r < RP; ++r)
          if (r == my_r) mrow = m_new[r];
        const float p = (sc == -INFINITY) ? 0.f : exp2f(sc - mrow);
        float ps = p;
#pragma unroll
        for (int off = RP << SHIFT; off < 32; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
        if ((lane & ((1 << SHIFT) - 1)) == 0) pbuf[warp * 32 + my_idx] = p;
#pragma unroll
        for (int r = 0; r < RP; ++r) {
          const float step_sum = __shfl_sync(0xffffffffu, ps, r << SHIFT);
          const float corr = (m_run[r] == -INFINITY) ? 0.f : exp2f(m_run[r] - m_new[r]);
          l_run[r] = l_run[r] * corr + step_sum;
          m_run[r] = m_new[r];
#pragma unroll
          for (int e = 0; e < EPL; ++e) o[r][e] *= corr;
        }
        __syncwarp();
#pragma unroll
        for (int kk = 0; kk < KWW; ++kk) {
          const int kl = kl0 + kk;
          const T* vr = vt + (size_t)kl * D + lane * EPL;
          float vf[EPL];
#pragma unroll
          for (int e = 0; e < EPL; ++e) vf[e] = (j0 + kl < kend) ? to_f<T>(vr[e]) : 0.f;
#pragma unroll
          for (int r = 0; r < RP; ++r) {
            const float pr = pbuf[warp * 32 + kk * RP + r];
#pragma unroll
            for (int e = 0; e < EPL; ++e) o[r][e] = fmaf(pr, vf[e], o[r][e]);
          }
        }
        __syncwarp();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int r = 0; r < RP; ++r) {
      float* w = wst + ((size_t)warp * RP + r) * (D + 2);
#pragma unroll
      for (int e = 0; e < EPL; ++e) w[lane * EPL + e] = o[r][e];
      if (lane == 0) {
        w[D] = m_run[r];
        w[D + 1] = l_run[r];
      }
    }
  }
  __syncthreads();
  if (flags[0] && threadIdx.x == 0) {
    report_device_error(kp.err, kErrGqaTimeout, blockIdx.x);
    // let the copies still in flight land before this CTA's shared memory is released
    for (int t = flags[3]; t < flags[2]; ++t) mbar_wait(&full[t % stages], (t / stages) & 1, 1u << 20);
  }
  __syncthreads();

  // --- merge the warps; write the output or this split's partial -----------------------------
  float* part = kp.partial + ((((int64_t)b * kp.HK + kvh) * kp.splits + split) * RP) * (D + 2);
  for (int idx = threadIdx.x; idx < kp.R * (D + 2); idx += kThreads) {
    const int r = idx / (D + 2), d = idx - r * (D + 2);
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kNW; ++w) M = fmaxf(M, wst[((size_t)w * RP + r) * (D + 2) + D]);
    float acc = 0.f, lsum = 0.f;
#pragma unroll
    for (int w = 0; w < kNW; ++w) {
      const float* ws = wst + ((size_t)w * RP + r) * (D + 2);
      const float f = (ws[D] == -INFINITY) ? 0.f : exp2f(ws[D] - M);
      if (d < D) acc = fmaf(ws[d], f, acc);
      lsum = fmaf(ws[D + 1], f, lsum);
    }
    if (kp.splits == 1) {
      if (d < D) {
        const int s = r / kp.G, g = r - s * kp.G, h = kvh * kp.G + g;
        T* out = static_cast<T*>(kp.out) + (((int64_t)b * kp.S + s) * kp.H + h) * D;
        out[d] = from_f<T>(lsum > 0.f ? acc / lsum : 0.f);
      }
    } else {
      part[idx] = d < D ? acc : (d == D ? M : lsum);
    }
  }
  if (kp.splits == 1) return;

  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int ticket = atomicAdd(&kp.counters[b * kp.HK + kvh], 1);
    flags[1] = (ticket == kp.splits - 1);
  }
  __syncthreads();
  if (!flags[1]) return;
  __threadfence();
  // --- last CTA of this (batch, kv-head): merge the splits ---------------------------------
  // per-(split, row) weights first (one pass over the small m / l vectors), then every output
  // element sums its splits with independent loads.
  const float* base = kp.partial + (((int64_t)b * kp.HK + kvh) * kp.splits) * RP * (D + 2);
  float* wsp = reinterpret_cast<float*>(smem + L.kbuf);  // [splits][RP] weights (tile buffers are free)
  float* rowM = wsp + kp.splits * RP;                     // [RP]
  for (int i = threadIdx.x; i < kp.splits * kp.R; i += kThreads) {
    const int sp = i / kp.R, r = i - sp * kp.R;
    wsp[sp * RP + r] = __ldcg(base + ((size_t)sp * RP + r) * (D + 2) + D);  // m
  }
  __syncthreads();
  if (threadIdx.x < kp.R) {
    const int r = threadIdx.x;
    float M = -INFINITY;
    for (int sp = 0; sp < kp.splits; ++sp) M = fmaxf(M, wsp[sp * RP + r]);
    float lsum = 0.f;
    for (int sp = 0; sp < kp.splits; ++sp) {
      const float m = wsp[sp * RP + r];
      const float f = (m == -INFINITY) ? 0.f : exp2f(m - M);
      wsp[sp * RP + r] = f;
      lsum = fmaf(__ldcg(base + ((size_t)sp * RP + r) * (D + 2) + D + 1), f, lsum);
    }
    rowM[r] = lsum > 0.f ? 1.f / lsum : 0.f;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < kp.R * D; idx += kThreads) {
    const int r = idx / D, d = idx - r * D;
    float acc = 0.f;
    int sp = 0;
    for (; sp + 4 <= kp.splits; sp += 4) {
      const float a0 = __ldcg(base + ((size_t)(sp + 0) * RP + r) * (D + 2) + d);
      const float a1 = __ldcg(base + ((size_t)(sp + 1) * RP + r) * (D + 2) + d);
      const float a2 = __ldcg(base + ((size_t)(sp + 2) * RP + r) * (D + 2) + d);
      const float a3 = __ldcg(base + ((size_t)(sp + 3) * RP + r) * (D + 2) + d);
      acc = fmaf(a0, wsp[(sp + 0) * RP + r], acc);
      acc = fmaf(a1, wsp[(sp + 1) * RP + r], acc);
      acc = fmaf(a2, wsp[(sp + 2) * RP + r], acc);
      acc = fmaf(a3, wsp[(sp + 3) * RP + r], acc);
    }
    for (; sp < kp.splits; ++sp) acc = fmaf(__ldcg(base + ((size_t)sp * RP + r) * (D + 2) + d), wsp[sp * RP + r], acc);
    const int s = r / kp.G, g = r - s * kp.G, h = kvh * kp.G + g;
    T* out = static_cast<T*>(kp.out) + (((int64_t)b * kp.S + s) * kp.H + h) * D;
    out[d] = from_f<T>(acc * rowM[r]);
  }
  if (threadIdx.x == 0) kp.counters[b * kp.HK + kvh] = 0;
}

// ---- generic path ---------------------------------------------------------------------------
// One warp per new row: q rows (H per token) go to kp.qrot (fp32, rounded through T); k rows are
// rotated and written with v into the KV buffer.
template <typename T>
__global__ void gqa_append_kernel(GqaKP kp) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float rowbuf[];  // [warps][D]
  const int warps = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_tok = kp.H + kp.HK;
  const int item = blockIdx.x * warps + warp;
  if (item >= kp.B * kp.S * per_tok) return;
  const int b = item / (kp.S * per_tok);
  const int rem = item - b * kp.S * per_tok;
  const int s = rem / per_tok, hh = rem - s * per_tok;
  const int past = past_len(kp, b);
  if (!range_ok(kp, past)) {
    if (lane == 0) report_device_error(kp.err, kErrGqaRange, b);
    return;
  }
  const int pos = past + s;
  const int D = kp.D;
  float* row = rowbuf + warp * D;
  if (hh < kp.H) {
    const T* src = static_cast<const T*>(kp.q) + ((int64_t)b * kp.S + s) * kp.qstride + (int64_t)hh * D;
    for (int i = lane; i < D; i += 32) row[i] = to_f<T>(src[i]);
    __syncwarp();
    rotate_row_warp<T>(row, D, pos, kp, kp.qn);
    float* dst = kp.qrot + (((int64_t)b * kp.S + s) * kp.H + hh) * D;
    for (int i = lane; i < D; i += 32) dst[i] = row[i];
  } else {
    const int kvh = hh - kp.H;
    const int64_t in_off = ((int64_t)b * kp.S + s) * kp.kstride + (int64_t)kvh * D;
    const T* kin = static_cast<const T*>(kp.k);
    const T* vin = static_cast<const T*>(kp.v);
    for (int i = lane; i < D; i += 32) row[i] = to_f<T>(kin[in_off + kp.koff + i]);
    __syncwarp();
    rotate_row_warp<T>(row, D, pos, kp, kp.kn);
    const int64_t dst = (((int64_t)b * kp.HK + kvh) * kp.cap + pos) * D;
    T* kvk = static_cast<T*>(kp.kv_k);
    T* kvv = static_cast<T*>(kp.kv_v);
    for (int i = lane; i < D; i += 32) {
      kvk[dst + i] = from_f<T>(row[i]);
      kvv[dst + i] = vin[in_off + kp.voff + i];
    }
  }
}

// One CTA (128 threads) per (b, s, h) query row; scores for all keys staged in shared memory.
template <typename T>
__global__ void __launch_bounds__(128) gqa_generic_kernel(GqaKP kp) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float sh[];  // [D] q, [cap] scores, [4] reduction
  const int row = blockIdx.x;
  const int h = row % kp.H, s = (row / kp.H) % kp.S, b = row / (kp.H * kp.S);
  const int past = past_len(kp, b);
  if (!range_ok(kp, past)) return;
  const int D = kp.D, kvh = h / kp.G;
  const int qpos = past + s;
  const int lo = kp.local_window > 0 ? max(0, qpos - kp.local_window + 1) : 0;
  const int n = qpos + 1 - lo;
  float* qv = sh;
  float* sc = sh + D;
  float* red = sc + kp.cap;
  const float* qsrc = kp.qrot + (((int64_t)b * kp.S + s) * kp.H + h) * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) qv[i] = qsrc[i];
  __syncthreads();
  const T* kc = static_cast<const T*>(kp.kv_k) + ((int64_t)b * kp.HK + kvh) * kp.cap * D;
  const T* vc = static_cast<const T*>(kp.kv_v) + ((int64_t)b * kp.HK + kvh) * kp.cap * D;
  const T* bias = static_cast<const T*>(kp.bias);
  float mx = -INFINITY;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    const int j = lo + t;
    float acc = 0.f;
    for (int i = 0; i < D; ++i) acc = fmaf(qv[i], to_f<T>(kc[(int64_t)j * D + i]), acc);
    float x = acc * kp.scale_log2;
    if (bias && j < kp.bias_total)
      x += to_f<T>(bias[((int64_t)(kp.bias_batch == 1 ? 0 : b) * kp.S + s) * kp.bias_total + j]) * kLog2e;
    sc[t] = x;
    mx = fmaxf(mx, x);
  }
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  float sum = 0.f;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    const float p = exp2f(sc[t] - mx);
    sc[t] = p;
    sum += p;
  }
  sum = warp_sum(sum);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  sum = red[0] + red[1] + red[2] + red[3];
  T* out = static_cast<T*>(kp.out) + (((int64_t)b * kp.S + s) * kp.H + h) * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float acc = 0.f;
    for (int t = 0; t < n; ++t) acc = fmaf(sc[t], to_f<T>(vc[(int64_t)(lo + t) * D + i]), acc);
    out[i] = from_f<T>(sum > 0.f ? acc / sum : 0.f);
  }
}

// ---- host side ------------------------------------------------------------------------------

// ---- tensor-core decode kernel ---------------------------------------------------------------
// gqa_mma_decode_kernel — one query row per sequence (S == 1), G <= 8 query heads per KV head,
// head_size 64 or 128, fp16 / bf16.  grid (splits, kv_heads, batch) with the splits of one
// (batch, kv-head) in one thread-block cluster; 4 warps per CTA.
//   * The keys [lo, past] are cut into 32-key units spread over the splits x 4 warps of the
//     cluster.  Each warp streams its units through two shared-memory buffers with 16-byte
//     cp.async copies (rows XOR-swizzled so ldmatrix reads are conflict-free).
//   * S = Q K^T and O += P V run on mma.sync.m16n8k16 (fp32 accumulate): the G rotated query rows
//     are the A operand (rows G..15 zero), K and V reach the B operand through ldmatrix /
//     ldmatrix.trans, and the probabilities go from the score accumulators straight into the A
//     fragments of P V.  Online softmax in base 2, fp32.
//   * The warp that owns the newest key (position past) rotates the new k row, writes k and v into
//     the KV buffer and patches its shared-memory copy of that unit (the copy it streamed may
//     predate the append).
//   * Warps merge in shared memory; the CTAs of the cluster merge through distributed shared memory
//     into the output (no workspace, no second pass).
constexpr int kMmaWarps = 4;
constexpr int kUnit = 32;  // keys per unit

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_addr(p)));
}

template <typename T>
__device__ __forceinline__ void mma_f32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value)
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  T a = from_f<T>(lo), b = from_f<T>(hi);
  uint16_t ua, ub;
  memcpy(&ua, &a, 2);
  memcpy(&ub, &b, 2);
  return (uint32_t)ua | ((uint32_t)ub << 16);
}

// byte offset of 16-byte chunk `ch` of row `r` in a swizzled [rows][D] tile
template <int D>
__device__ __forceinline__ int swz(int r, int ch) {
  return r * D * 2 + ((ch ^ (r & 7)) << 4);
}

template <int D>
struct MmaSmem {
  static constexpr int kUnitBytes = kUnit * D * 2;            // one K (or V) unit
  static constexpr int kBufs = 3;                              // units in flight per warp
  static constexpr int kWarpBytes = kBufs * 2 * kUnitBytes;    // buffers x (K, V)
  static constexpr int kQStride = D + 8;                      // halves, padded
  static constexpr int kQ = kMmaWarps * kWarpBytes;           // [16][kQStride] halves
  static constexpr int kScratch = kQ + 16 * kQStride * 2;     // [kMmaWarps][D] floats
  static constexpr int kMerge = kScratch + kMmaWarps * D * 4; // [8][D + 2] floats (CTA result)
  static constexpr int kTotal = kMerge + 8 * (D + 2) * 4;
};

// The sequence of packed row i (cum[b] <= i < cum[b + 1]) or -1, and the cache row of its key j or -1.
__device__ __forceinline__ int paged_seq(const GqaKP& kp, int i) {
  int lo = 0, hi = kp.p_batch;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(kp.p_cum + mid) <= i) lo = mid;
    else hi = mid - 1;
  }
  if (lo >= kp.p_batch || __ldg(kp.p_cum + lo) > i || i >= __ldg(kp.p_cum + lo + 1)) return -1;
  return lo;
}
__device__ __forceinline__ int paged_row(const GqaKP& kp, int seq, int j) {
  const int blk = j / kp.p_bs;
  if (j < 0 || blk >= kp.p_maxb) return -1;
  const int phys = __ldg(kp.p_bt + (size_t)seq * kp.p_maxb + blk);
  return phys < 0 || phys >= kp.p_nblocks ? -1 : phys * kp.p_bs + j % kp.p_bs;
}

// PAGED: the PagedAttention form (see GqaKP); the new rows were appended by a preceding launch, so
// the K / V stream starts after the wait for it and no warp appends.
template <typename T, int D, bool PAGED = false>
__global__ void __launch_bounds__(kMmaWarps * 32)
gqa_mma_decode_kernel(GqaKP kp) {
  using L = MmaSmem<D>;
  constexpr int NB = D / 8;   // 8-wide n-blocks of the output
  constexpr int KS = D / 16;  // k-steps of q.k
  extern __shared__ __align__(128) unsigned char sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int kvh = blockIdx.y, b = blockIdx.z;
  uint32_t crank, csize;
  asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
  asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(csize));

  // Before the wait: everything that depends only on data written two or more kernels back —
  // the positions (seqlens), the KV rows of earlier steps and the rotary tables (see pdl_trigger).
  int past;
  bool ok;
  int pseq = -1;  // PAGED: the row's sequence
  if constexpr (PAGED) {
    pseq = paged_seq(kp, b);
    past = pseq >= 0 ? __ldg(kp.p_past + pseq) + (b - __ldg(kp.p_cum + pseq)) : -1;
    ok = past >= 0 && (!kp.do_rotary || past < kp.max_seq);
  } else {
    past = past_len(kp, b);
    ok = range_ok(kp, past);
  }
  const int nk = ok ? past + 1 : 0;  // keys [lo, nk)
  const int lo = kp.local_window > 0 ? max(0, past - kp.local_window + 1) : 0;
  const int units = nk > lo ? (nk - lo + kUnit - 1) / kUnit : 0;
  const int nw = (int)csize * kMmaWarps, wid = (int)crank * kMmaWarps + warp;
  const int u0 = (int)((int64_t)units * wid / nw), u1 = (int)((int64_t)units * (wid + 1) / nw);
  const int64_t head_base = ((int64_t)b * kp.HK + kvh) * kp.cap;
  T* kvk = static_cast<T*>(kp.kv_k) + head_base * D;
  T* kvv = static_cast<T*>(kp.kv_v) + head_base * D;

  unsigned char* wbuf = sm + warp * L::kWarpBytes;  // [buf][K | V]
  bool bad_row = false;  // PAGED: a key row outside the caches (read as zeros, reported)
  // PAGED: lane l holds the cache row of key l of the next unit to issue; each issue uses it and
  // starts the block-table load of the unit after, so that lookup overlaps a whole unit.  (The
  // block table is not written by the kernels before this one, so the first lookup may precede
  // the programmatic-launch wait.)
  auto lookup = [&](int u) {
    const int j = lo + u * kUnit + lane;
    return j < nk ? paged_row(kp, pseq, j) : -1;
  };
  int prow_next = 0;
  if constexpr (PAGED) prow_next = lookup(u0);
  auto issue = [&](int u, int buf) {
    unsigned char* kb = wbuf + buf * 2 * L::kUnitBytes;
    unsigned char* vb = kb + L::kUnitBytes;
    const int key0 = lo + u * kUnit;
    if constexpr (PAGED) {
      // lane l looked up the cache row of key key0 + l; the copies take it by shuffle
      const int prow = prow_next;
      prow_next = lookup(u + 1);
      bad_row |= key0 + lane < nk && prow < 0;
      const T* kc = static_cast<const T*>(kp.kv_k);
      const T* vc = static_cast<const T*>(kp.kv_v);
      for (int i = lane; i < kUnit * D / 8; i += 32) {
        const int r = i / (D / 8), ch = i % (D / 8);
        const int pr = __shfl_sync(0xffffffffu, prow, r);
        const bool v = pr >= 0;
        const int64_t off = v ? ((int64_t)pr * kp.HK + kvh) * D + ch * 8 : 0;
        cp_async16(kb + swz<D>(r, ch), kc + off, v);
        cp_async16(vb + swz<D>(r, ch), vc + off, v);
      }
    } else {
      for (int i = lane; i < kUnit * D / 8; i += 32) {
        const int r = i / (D / 8), ch = i % (D / 8);
        const bool v = key0 + r < nk;
        const int64_t row = v ? key0 + r : 0;
        cp_async16(kb + swz<D>(r, ch), kvk + row * D + ch * 8, v);
        cp_async16(vb + swz<D>(r, ch), kvv + row * D + ch * 8, v);
      }
    }
    cp_async_commit();
  };
  if constexpr (!PAGED)
    for (int k = 0; k < L::kBufs; ++k)
      if (u0 + k < u1) issue(u0 + k, k);
  float cs[4] = {0, 0, 0, 0}, sn[4] = {0, 0, 0, 0};  // rotary pairs i = lane + 32 * e of this position
  if (ok && kp.do_rotary) {
    const T* cc = static_cast<const T*>(kp.cos_c) + (int64_t)past * kp.half;
    const T* sc = static_cast<const T*>(kp.sin_c) + (int64_t)past * kp.half;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (lane + 32 * e < kp.half) cs[e] = to_f<T>(cc[lane + 32 * e]), sn[e] = to_f<T>(sc[lane + 32 * e]);
  }
  // one head row (fp32 in shared memory) through the optional per-head RMS norm and RoPE, rounded
  // through T as stored — the arithmetic of rotate_row_warp with the tables preloaded
  auto rotate = [&](float* row, const void* normw) {
    if (kp.has_qk_norm) {
      float ss = 0.f;
      for (int i = lane; i < D; i += 32) ss = fmaf(row[i], row[i], ss);
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / (float)D + kp.qk_eps);
      const T* w = static_cast<const T*>(normw);
      for (int i = lane; i < D; i += 32) row[i] = row[i] * inv * to_f<T>(w[i]);
      __syncwarp();
    }
    if (kp.do_rotary) {
      float o0[4], o1[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = lane + 32 * e;
        if (i < kp.half) {
          const int i0 = kp.interleaved ? 2 * i : i;
          const int i1 = kp.interleaved ? 2 * i + 1 : i + kp.half;
          const float a = row[i0], bb = row[i1];
          o0[e] = a * cs[e] - bb * sn[e];
          o1[e] = bb * cs[e] + a * sn[e];
        }
      }
      __syncwarp();
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = lane + 32 * e;
        if (i < kp.half) {
          row[kp.interleaved ? 2 * i : i] = o0[e];
          row[kp.interleaved ? 2 * i + 1 : i + kp.half] = o1[e];
        }
      }
      __syncwarp();
    }
    for (int i = lane; i < D; i += 32) row[i] = round_through<T>(row[i]);
    __syncwarp();
  };

  pdl_wait();  // q / k / v come from the previous kernel
  pdl_trigger();
  if constexpr (PAGED)  // the previous launch appended this step's rows
    for (int k = 0; k < L::kBufs; ++k)
      if (u0 + k < u1) issue(u0 + k, k);
  if (!ok && threadIdx.x == 0 && crank == 0 && kvh == 0) report_device_error(kp.err, kErrGqaRange, b);

  // rotated query rows (rounded through T, as stored) -> Qs rows 0..G-1; rows G..15 zero
  T* Qs = reinterpret_cast<T*>(sm + L::kQ);
  float* scratch = reinterpret_cast<float*>(sm + L::kScratch) + warp * D;
  for (int i = threadIdx.x; i < (16 - kp.G) * L::kQStride; i += kMmaWarps * 32)
    Qs[kp.G * L::kQStride + i] = from_f<T>(0.f);
  // the owner of the newest key appends it: rotated k and v into the KV buffer (and, below, into
  // its streamed copy of that unit, which was read before the append).  Its k / v loads are issued
  // together with the query loads, so the two round trips overlap.
  const int u_new = nk > lo ? (nk - 1 - lo) / kUnit : -1;
  const bool owner = !PAGED && ok && u_new >= u0 && u_new < u1;
  T knew[D / 32], vnew[D / 32], kraw[D / 32];
  const int64_t in_off = (int64_t)b * kp.kstride + (int64_t)kvh * D;
  if (owner) {
    const T* kin = static_cast<const T*>(kp.k);
    const T* vin = static_cast<const T*>(kp.v);
#pragma unroll
    for (int e = 0; e < D / 32; ++e) {
      kraw[e] = kin[in_off + kp.koff + lane + 32 * e];
      vnew[e] = vin[in_off + kp.voff + lane + 32 * e];
    }
  }
  if (ok) {
    const T* qin = static_cast<const T*>(kp.q);
    for (int gq = warp; gq < kp.G; gq += kMmaWarps) {
      const T* src = qin + (int64_t)b * kp.qstride + (int64_t)(kvh * kp.G + gq) * D;
      // D / 32 consecutive values per lane in one load
      if constexpr (D == 128) {
        const uint2 w = *reinterpret_cast<const uint2*>(src + lane * 4);
        const T* h = reinterpret_cast<const T*>(&w);
#pragma unroll
        for (int e = 0; e < 4; ++e) scratch[lane * 4 + e] = to_f<T>(h[e]);
      } else {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(src + lane * 2);
        const T* h = reinterpret_cast<const T*>(&w);
#pragma unroll
        for (int e = 0; e < 2; ++e) scratch[lane * 2 + e] = to_f<T>(h[e]);
      }
      __syncwarp();
      rotate(scratch, kp.qn);
      for (int i = lane; i < D; i += 32) Qs[gq * L::kQStride + i] = from_f<T>(scratch[i]);
      __syncwarp();
    }
  }
  if (owner) {
#pragma unroll
    for (int e = 0; e < D / 32; ++e) scratch[lane + 32 * e] = to_f<T>(kraw[e]);
    __syncwarp();
    rotate(scratch, kp.kn);
#pragma unroll
    for (int e = 0; e < D / 32; ++e) {
      const int i = lane + 32 * e;
      knew[e] = from_f<T>(scratch[i]);
      kvk[(int64_t)past * D + i] = knew[e];
      kvv[(int64_t)past * D + i] = vnew[e];
    }
  }
  __syncthreads();

  // Q as A fragments, one per k-step
  uint32_t qa[KS][4];
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) {
    const int row = (lane & 7) + ((lane >> 3) & 1) * 8, col = kk * 16 + (lane >> 4) * 8;
    ldsm_x4(qa[kk], Qs + row * L::kQStride + col);
  }

  float m_run = -INFINITY, l_run = 0.f;  // row g (lanes with g < G hold real rows)
  float o[NB][4];
#pragma unroll
  for (int n = 0; n < NB; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  const T* bias = static_cast<const T*>(kp.bias);
  const int64_t bias_row = kp.bias_batch > 0 ? (int64_t)(kp.bias_batch == 1 ? 0 : b) * kp.bias_total : 0;

  for (int u = u0; u < u1; ++u) {
    const int buf = (u - u0) % L::kBufs;
    if (u + 2 < u1) cp_async_wait<2>();
    else if (u + 1 < u1) cp_async_wait<1>();
    else cp_async_wait<0>();
    __syncwarp();
    unsigned char* kb = wbuf + buf * 2 * L::kUnitBytes;
    unsigned char* vb = kb + L::kUnitBytes;
    const int key0 = lo + u * kUnit;
    if (owner && u == u_new) {
      const int r = nk - 1 - key0;
#pragma unroll
      for (int e = 0; e < D / 32; ++e) {
        const int i = lane + 32 * e;
        *reinterpret_cast<T*>(kb + swz<D>(r, i >> 3) + (i & 7) * 2) = knew[e];
        *reinterpret_cast<T*>(vb + swz<D>(r, i >> 3) + (i & 7) * 2) = vnew[e];
      }
      __syncwarp();
    }
    // S = Q K^T for the unit's 32 keys: 4 n-blocks of 8 keys
    float sacc[4][4];
#pragma unroll
    for (int nb = 0; nb < 4; ++nb) {
      sacc[nb][0] = sacc[nb][1] = sacc[nb][2] = sacc[nb][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < KS; kk += 2) {
        uint32_t bfr[4];
        ldsm_x4(bfr, kb + swz<D>(nb * 8 + (lane & 7), kk * 2 + (lane >> 3)));
        mma_f32<T>(sacc[nb], qa[kk], bfr[0], bfr[1]);
        mma_f32<T>(sacc[nb], qa[kk + 1], bfr[2], bfr[3]);
      }
    }
    // scores of row g for keys key0 + nb*8 + 2c (+1); online softmax in base 2
    float sc[4][2], mx = -INFINITY;
#pragma unroll
    for (int nb = 0; nb < 4; ++nb)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = key0 + nb * 8 + 2 * c + h;
        float v = sacc[nb][h] * kp.scale_log2;
        if (bias && j < kp.bias_total) v += to_f<T>(bias[bias_row + j]) * kLog2e;
        v = j < nk ? v : -INFINITY;
        sc[nb][h] = v;
        mx = fmaxf(mx, v);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float corr = m_run == -INFINITY ? 0.f : exp2f(m_run - m_new);
    float ps = 0.f;
    uint32_t pa[2][4];  // P as A fragments for the two 16-key k-steps (rows g+8 zero)
    // PagedAttention in bf16: P as hi + lo bf16 parts (two P.V MMAs), since its rows with few keys
    // have large probabilities whose 8-bit rounding would show in the output
    constexpr bool kPSplit = PAGED && std::is_same<T, __nv_bfloat16>::value;
    uint32_t pl[2][4];
#pragma unroll
    for (int nb = 0; nb < 4; ++nb) {
      const float p0 = sc[nb][0] == -INFINITY ? 0.f : exp2f(sc[nb][0] - m_new);
      const float p1 = sc[nb][1] == -INFINITY ? 0.f : exp2f(sc[nb][1] - m_new);
      ps += p0 + p1;
      pa[nb >> 1][(nb & 1) * 2] = pack2<T>(p0, p1);
      pa[nb >> 1][(nb & 1) * 2 + 1] = 0u;
      if constexpr (kPSplit) {
        pl[nb >> 1][(nb & 1) * 2] = pack2<T>(p0 - round_through<T>(p0), p1 - round_through<T>(p1));
        pl[nb >> 1][(nb & 1) * 2 + 1] = 0u;
      }
    }
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    l_run = l_run * corr + ps;
    m_run = m_new;
    if (!__all_sync(0xffffffffu, corr == 1.f)) {
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        o[n][0] *= corr;
        o[n][1] *= corr;
      }
    }
    // O += P V
#pragma unroll
    for (int ks = 0; ks < 2; ++ks)
#pragma unroll
      for (int n = 0; n < NB; n += 2) {
        uint32_t bfr[4];
        const int r = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        ldsm_x4_t(bfr, vb + swz<D>(r, n + (lane >> 4)));
        mma_f32<T>(o[n], pa[ks], bfr[0], bfr[1]);
        mma_f32<T>(o[n + 1], pa[ks], bfr[2], bfr[3]);
        if constexpr (kPSplit) {
          mma_f32<T>(o[n], pl[ks], bfr[0], bfr[1]);
          mma_f32<T>(o[n + 1], pl[ks], bfr[2], bfr[3]);
        }
      }
    __syncwarp();
    if (u + L::kBufs < u1) issue(u + L::kBufs, buf);
  }

  if constexpr (PAGED)
    if (__any_sync(0xffffffffu, bad_row) && lane == 0) report_device_error(kp.err, kErrGqaRange, b);
  // merge the warps: per-warp (m, l, O) rows into shared memory (reusing the stream buffers)
  __syncthreads();
  float* wst = reinterpret_cast<float*>(sm);  // [kMmaWarps][8][D + 2]
  if (g < kp.G) {
    float* row = wst + ((size_t)warp * 8 + g) * (D + 2);
#pragma unroll
    for (int n = 0; n < NB; ++n) {
      row[n * 8 + 2 * c] = o[n][0];
      row[n * 8 + 2 * c + 1] = o[n][1];
    }
    if (c == 0) {
      row[D] = m_run;
      row[D + 1] = l_run;
    }
  }
  __syncthreads();
  float* res = reinterpret_cast<float*>(sm + L::kMerge);  // [8][D + 2]: this CTA's (O, m, l)
  for (int i = threadIdx.x; i < kp.G * (D + 2); i += kMmaWarps * 32) {
    const int gq = i / (D + 2), d = i - gq * (D + 2);
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kMmaWarps; ++w) M = fmaxf(M, wst[((size_t)w * 8 + gq) * (D + 2) + D]);
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kMmaWarps; ++w) {
      const float* row = wst + ((size_t)w * 8 + gq) * (D + 2);
      const float f = row[D] == -INFINITY ? 0.f : exp2f(row[D] - M);
      acc += (d < D ? row[d] : row[D + 1]) * f;
    }
    res[i] = d == D ? M : acc;  // O (unnormalised), m, l
  }
  // merge the cluster's CTAs through distributed shared memory: rank r writes outputs
  // [r * per, (r + 1) * per) of the G x D head rows, reading every rank's (O, m, l) for them
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (ok) {
    T* out = static_cast<T*>(kp.out) + (int64_t)b * kp.H * D + (int64_t)kvh * kp.G * D;
    const uint32_t local = smem_addr(res);
    const int total = kp.G * D, per = (total + (int)csize - 1) / (int)csize;
    for (int i = (int)crank * per + threadIdx.x; i < min(total, ((int)crank + 1) * per); i += kMmaWarps * 32) {
      const int gq = i / D, d = i - gq * D;
      const uint32_t row = local + (uint32_t)(gq * (D + 2) * 4);
      float m[8], l[8], ov[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        m[r] = -INFINITY, l[r] = 0.f, ov[r] = 0.f;
        if (r < (int)csize) {
          uint32_t ra;
          asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(row), "r"(r));
          asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(ov[r]) : "r"(ra + (uint32_t)(d * 4)));
          asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(m[r]) : "r"(ra + (uint32_t)(D * 4)));
          asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(l[r]) : "r"(ra + (uint32_t)((D + 1) * 4)));
        }
      }
      float M = -INFINITY;
#pragma unroll
      for (int r = 0; r < 8; ++r) M = fmaxf(M, m[r]);
      float num = 0.f, den = 0.f;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float f = m[r] == -INFINITY ? 0.f : exp2f(m[r] - M);
        num += ov[r] * f;
        den += l[r] * f;
      }
      out[(int64_t)gq * D + d] = from_f<T>(den > 0.f ? num / den : 0.f);
    }
  }
  // keep every CTA's shared memory alive until all ranks have read it
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---- tensor-core prefill kernel --------------------------------------------------------------
// gqa_mma_prefill_kernel — S > 1 (prompt) attention after gqa_append_kernel has rotated the query
// rows into the fp32 workspace (rounded through T) and written the rotated k and v rows into the
// KV buffer.  grid (ceil(S / 64), num_heads, batch), 4 warps; warp w owns query rows
// [64 x + 16 w, + 16).  Key tiles of 64 keys x D stream through two shared-memory buffers by
// 16-byte cp.async (rows XOR-swizzled for conflict-free ldmatrix); S = Q K^T and O += P V run on
// mma.sync.m16n8k16 with fp32 accumulation and a base-2 online softmax per row; the tile loop
// stops at the block's last causal key and starts at its first windowed key.  Query i (position
// past + i) sees keys [lo_i, past + i] — the bottom-right-aligned causal mask of ONNX GQA.
// (Measured alternatives, slower on B200 except at prompts of 4K and more: 8 warps per CTA sharing
// each K / V tile, and 32-key tiles with the Q fragments re-read from shared memory for four CTAs
// per SM.  mma.sync bounds this kernel; the tcgen05 form is the next step.)
constexpr int kPfWarps = 4;
constexpr int kPfRows = 16 * kPfWarps;  // query rows per CTA
constexpr int kPfKeys = 64;             // keys per tile

template <int D>
struct PfSmem {
  static constexpr int kTile = kPfKeys * D * 2;  // one K or V tile
  static constexpr int kTotal = 2 * 2 * kTile;   // [buffer][K, V]
};

// PAGED: the PagedAttention form (see GqaKP): blockIdx.z is a sequence whose rows are the packed
// rows [p_cum[b], p_cum[b + 1]) of kp.S; the preceding append launch wrote their rotated q rows
// (rounded to T) into the output rows, which each CTA reads before it overwrites them; key tiles
// take their row addresses from the block table, looked up one tile ahead.
template <typename T, int D, bool PAGED = false>
__global__ void __launch_bounds__(kPfWarps * 32)
gqa_mma_prefill_kernel(GqaKP kp) {
  using L = PfSmem<D>;
  constexpr int NB = D / 8;   // 8-wide n-blocks of O
  constexpr int KS = D / 16;  // k-steps of q.k
  extern __shared__ __align__(128) unsigned char sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int h = blockIdx.y, b = blockIdx.z, kvh = h / kp.G;
  int past, Sb;       // past length and rows of this sequence
  int64_t row0 = 0;   // PAGED: its first packed row
  if constexpr (PAGED) {
    row0 = __ldg(kp.p_cum + b);
    Sb = __ldg(kp.p_cum + b + 1) - (int)row0;
    past = __ldg(kp.p_past + b);
    if (Sb <= 0 || row0 < 0 || row0 + Sb > kp.S || past < 0 || (kp.do_rotary && past + Sb > kp.max_seq)) return;
  } else {
    past = past_len(kp, b);
    Sb = kp.S;
    if (!range_ok(kp, past)) return;  // reported by gqa_append_kernel
  }
  const int i0 = blockIdx.x * kPfRows;
  if (PAGED && i0 >= Sb) return;
  const int ilast = min(Sb, i0 + kPfRows) - 1;  // last query row of the CTA
  const int win = kp.local_window;
  const int lo_blk = win > 0 ? max(0, past + i0 - win + 1) : 0;
  const int hi_blk = past + ilast;  // last key any row of the CTA sees
  const int t0 = lo_blk / kPfKeys, t1 = hi_blk / kPfKeys;
  const int64_t head_base = ((int64_t)b * kp.HK + kvh) * kp.cap;
  const T* kvk = static_cast<const T*>(kp.kv_k) + head_base * D;
  const T* kvv = static_cast<const T*>(kp.kv_v) + head_base * D;

  // PAGED: thread r < 64 holds the cache row of key r of the next tile to issue (looked up one tile
  // ahead; the block table is not written by the append, so the first lookup precedes the wait)
  __shared__ int prow_s[PAGED ? 2 : 1][PAGED ? kPfKeys : 1];
  bool bad_row = false;
  auto lookup = [&](int t) {
    const int j = t * kPfKeys + (int)threadIdx.x;
    return threadIdx.x < kPfKeys && j <= hi_blk ? paged_row(kp, b, j) : -1;
  };
  int prow_next = 0;
  if constexpr (PAGED) prow_next = lookup(t0);
  pdl_wait();  // the append kernel wrote the rotated q rows and the new k / v rows
  pdl_trigger();
  auto issue = [&](int t, int buf) {
    unsigned char* kb = sm + buf * 2 * L::kTile;
    unsigned char* vb = kb + L::kTile;
    const int key0 = t * kPfKeys;
    if constexpr (PAGED) {
      if (threadIdx.x < kPfKeys) {
        bad_row |= key0 + (int)threadIdx.x <= hi_blk && prow_next < 0;
        prow_s[buf][threadIdx.x] = prow_next;
      }
      prow_next = lookup(t + 1);
      __syncthreads();
      const T* kc = static_cast<const T*>(kp.kv_k);
      const T* vc = static_cast<const T*>(kp.kv_v);
      for (int i = threadIdx.x; i < kPfKeys * D / 8; i += kPfWarps * 32) {
        const int r = i / (D / 8), ch = i % (D / 8);
        const int pr = prow_s[buf][r];
        const bool v = pr >= 0;
        const int64_t off = v ? ((int64_t)pr * kp.HK + kvh) * D + ch * 8 : 0;
        cp_async16(kb + swz<D>(r, ch), kc + off, v);
        cp_async16(vb + swz<D>(r, ch), vc + off, v);
      }
    } else {
      for (int i = threadIdx.x; i < kPfKeys * D / 8; i += kPfWarps * 32) {
        const int r = i / (D / 8), ch = i % (D / 8);
        const bool v = key0 + r <= hi_blk;
        const int64_t row = v ? key0 + r : 0;
        cp_async16(kb + swz<D>(r, ch), kvk + row * D + ch * 8, v);
        cp_async16(vb + swz<D>(r, ch), kvv + row * D + ch * 8, v);
      }
    }
    cp_async_commit();
  };
  issue(t0, 0);

  // this lane's query rows ra = g and rb = g + 8 of the warp (index i, position past + i)
  const int ia = i0 + warp * 16 + g, ib = ia + 8;
  const bool va = ia < Sb, vb_ = ib < Sb;
  const int qa_pos = past + ia, qb_pos = past + ib;
  const int lo_a = win > 0 ? max(0, qa_pos - win + 1) : 0, lo_b = win > 0 ? max(0, qb_pos - win + 1) : 0;
  // Q as A fragments (the fp32 workspace holds values already rounded through T)
  uint32_t qf[KS][4];
  if constexpr (PAGED) {
    // the rotated rows (already T) in the output buffer
    const T* qo = static_cast<const T*>(kp.out);
    const T* qra = qo + ((row0 + (va ? ia : 0)) * kp.H + h) * D;
    const T* qrb = qo + ((row0 + (vb_ ? ib : 0)) * kp.H + h) * D;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      qf[kk][0] = va ? *reinterpret_cast<const uint32_t*>(qra + kk * 16 + 2 * c) : 0u;
      qf[kk][1] = vb_ ? *reinterpret_cast<const uint32_t*>(qrb + kk * 16 + 2 * c) : 0u;
      qf[kk][2] = va ? *reinterpret_cast<const uint32_t*>(qra + kk * 16 + 8 + 2 * c) : 0u;
      qf[kk][3] = vb_ ? *reinterpret_cast<const uint32_t*>(qrb + kk * 16 + 8 + 2 * c) : 0u;
    }
  } else {
    const float* qra = kp.qrot + (((int64_t)b * kp.S + (va ? ia : 0)) * kp.H + h) * D;
    const float* qrb = kp.qrot + (((int64_t)b * kp.S + (vb_ ? ib : 0)) * kp.H + h) * D;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      const float2 a0 = va ? *reinterpret_cast<const float2*>(qra + kk * 16 + 2 * c) : make_float2(0.f, 0.f);
      const float2 a1 = vb_ ? *reinterpret_cast<const float2*>(qrb + kk * 16 + 2 * c) : make_float2(0.f, 0.f);
      const float2 a2 = va ? *reinterpret_cast<const float2*>(qra + kk * 16 + 8 + 2 * c) : make_float2(0.f, 0.f);
      const float2 a3 = vb_ ? *reinterpret_cast<const float2*>(qrb + kk * 16 + 8 + 2 * c) : make_float2(0.f, 0.f);
      qf[kk][0] = pack2<T>(a0.x, a0.y);
      qf[kk][1] = pack2<T>(a1.x, a1.y);
      qf[kk][2] = pack2<T>(a2.x, a2.y);
      qf[kk][3] = pack2<T>(a3.x, a3.y);
    }
  }
  // rows of this warp: the first and last keys any of them sees
  const int wi0 = i0 + warp * 16, wi1 = min(Sb - 1, wi0 + 15);
  const int w_hi = past + wi1, w_lo = win > 0 ? max(0, past + wi0 - win + 1) : 0;

  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  float o[NB][4];
#pragma unroll
  for (int n = 0; n < NB; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

  for (int t = t0; t <= t1; ++t) {
    const int buf = (t - t0) & 1;
    if (t < t1) {
      issue(t + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int key0 = t * kPfKeys;
    // a warp whose rows all end before this tile (or start after it) skips it
    if (wi0 < Sb && key0 <= w_hi && key0 + kPfKeys - 1 >= w_lo) {
      const unsigned char* kb = sm + buf * 2 * L::kTile;
      const unsigned char* vb = kb + L::kTile;
      float sacc[8][4];
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
        sacc[nb][0] = sacc[nb][1] = sacc[nb][2] = sacc[nb][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < KS; kk += 2) {
          uint32_t bfr[4];
          ldsm_x4(bfr, kb + swz<D>(nb * 8 + (lane & 7), kk * 2 + (lane >> 3)));
          mma_f32<T>(sacc[nb], qf[kk], bfr[0], bfr[1]);
          mma_f32<T>(sacc[nb], qf[kk + 1], bfr[2], bfr[3]);
        }
      }
      // masks: key j is visible to row i iff lo_i <= j <= past + i
      const bool full = key0 >= max(lo_a, lo_b) && key0 + kPfKeys - 1 <= min(qa_pos, qb_pos) && va && vb_;
      float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
      for (int nb = 0; nb < 8; ++nb)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int j = key0 + nb * 8 + 2 * c + e;
          float sa = sacc[nb][e] * kp.scale_log2, sb = sacc[nb][2 + e] * kp.scale_log2;
          if (!full) {
            sa = (va && j >= lo_a && j <= qa_pos) ? sa : -INFINITY;
            sb = (vb_ && j >= lo_b && j <= qb_pos) ? sb : -INFINITY;
          }
          sacc[nb][e] = sa;
          sacc[nb][2 + e] = sb;
          mxa = fmaxf(mxa, sa);
          mxb = fmaxf(mxb, sb);
        }
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
      const float mna = fmaxf(m_a, mxa), mnb = fmaxf(m_b, mxb);
      const float ca = m_a == -INFINITY ? 0.f : exp2f(m_a - mna);
      const float cb = m_b == -INFINITY ? 0.f : exp2f(m_b - mnb);
      float psa = 0.f, psb = 0.f;
      uint32_t pa[4][4];  // P as A fragments for the tile's four 16-key k-steps
      // PagedAttention in bf16: P as hi + lo bf16 parts (see gqa_mma_decode_kernel)
      constexpr bool kPSplit = PAGED && std::is_same<T, __nv_bfloat16>::value;
      uint32_t pl[kPSplit ? 4 : 1][4];
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
        const float p0 = sacc[nb][0] == -INFINITY ? 0.f : exp2f(sacc[nb][0] - mna);
        const float p1 = sacc[nb][1] == -INFINITY ? 0.f : exp2f(sacc[nb][1] - mna);
        const float p2 = sacc[nb][2] == -INFINITY ? 0.f : exp2f(sacc[nb][2] - mnb);
        const float p3 = sacc[nb][3] == -INFINITY ? 0.f : exp2f(sacc[nb][3] - mnb);
        psa += p0 + p1;
        psb += p2 + p3;
        pa[nb >> 1][(nb & 1) * 2] = pack2<T>(p0, p1);
        pa[nb >> 1][(nb & 1) * 2 + 1] = pack2<T>(p2, p3);
        if constexpr (kPSplit) {
          pl[nb >> 1][(nb & 1) * 2] = pack2<T>(p0 - round_through<T>(p0), p1 - round_through<T>(p1));
          pl[nb >> 1][(nb & 1) * 2 + 1] = pack2<T>(p2 - round_through<T>(p2), p3 - round_through<T>(p3));
        }
      }
      psa += __shfl_xor_sync(0xffffffffu, psa, 1);
      psa += __shfl_xor_sync(0xffffffffu, psa, 2);
      psb += __shfl_xor_sync(0xffffffffu, psb, 1);
      psb += __shfl_xor_sync(0xffffffffu, psb, 2);
      l_a = l_a * ca + psa;
      l_b = l_b * cb + psb;
      m_a = mna;
      m_b = mnb;
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        o[n][0] *= ca;
        o[n][1] *= ca;
        o[n][2] *= cb;
        o[n][3] *= cb;
      }
      // O += P V
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
#pragma unroll
        for (int n = 0; n < NB; n += 2) {
          uint32_t bfr[4];
          const int r = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          ldsm_x4_t(bfr, vb + swz<D>(r, n + (lane >> 4)));
          mma_f32<T>(o[n], pa[ks], bfr[0], bfr[1]);
          mma_f32<T>(o[n + 1], pa[ks], bfr[2], bfr[3]);
          if constexpr (kPSplit) {
            mma_f32<T>(o[n], pl[ks], bfr[0], bfr[1]);
            mma_f32<T>(o[n + 1], pl[ks], bfr[2], bfr[3]);
          }
        }
    }
    __syncthreads();  // the buffer is refilled by the next iteration's prefetch
  }
  if constexpr (PAGED)
    if (__syncthreads_or(bad_row) && threadIdx.x == 0) report_device_error(kp.err, kErrGqaRange, b);

  T* out = static_cast<T*>(kp.out);
  const float ia_inv = l_a > 0.f ? 1.f / l_a : 0.f, ib_inv = l_b > 0.f ? 1.f / l_b : 0.f;
#pragma unroll
  for (int n = 0; n < NB; ++n) {
    if (va)
      *reinterpret_cast<uint32_t*>(out + ((PAGED ? row0 + ia : (int64_t)b * kp.S + ia) * kp.H + h) * D + n * 8 + 2 * c) =
          pack2<T>(o[n][0] * ia_inv, o[n][1] * ia_inv);
    if (vb_)
      *reinterpret_cast<uint32_t*>(out + ((PAGED ? row0 + ib : (int64_t)b * kp.S + ib) * kp.H + h) * D + n * 8 + 2 * c) =
          pack2<T>(o[n][2] * ib_inv, o[n][3] * ib_inv);
  }
}

namespace {

int pow2_at_least(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

bool decode_path(const b200ep_gqa_params& p, int esz) {
  const int G = (int)(p.num_heads / p.kv_heads);
  const int R = (int)(p.seq * G);
  return p.head_size % 32 == 0 && p.head_size <= 256 && R <= 32 &&
         pow2_at_least(R) * (p.head_size / 32) <= 64 && (p.head_size * esz) % 16 == 0;
}

int choose_splits(const b200ep_gqa_params& p) {
  const int64_t pairs = p.batch * p.kv_heads;
  int64_t want = (2 * 148 + pairs - 1) / pairs;
  int64_t max_by_len = std::max<int64_t>(1, p.cap / (2 * kKT));
  return (int)std::max<int64_t>(1, std::min<int64_t>({want, max_by_len, 64}));
}

struct WsLayout {
  size_t counters, partial, qrot, vt, base, total;  // base: without the optional V^T region
};

WsLayout ws_layout(const b200ep_gqa_params& p) {
  const int G = (int)(p.num_heads / p.kv_heads);
  const int RP = pow2_at_least((int)(p.seq * G));
  WsLayout w;
  size_t off = 0;
  w.counters = off;
  off += ((size_t)p.batch * p.kv_heads * sizeof(int) + 255) & ~(size_t)255;
  w.partial = off;
  // split-K partials exist only for decode-sized rows (the SIMT split-K kernel; decode_path)
  if (RP <= 32)
    off += ((size_t)p.batch * p.kv_heads * choose_splits(p) * RP * (p.head_size + 2) * 4 + 255) &
           ~(size_t)255;
  w.qrot = off;
  off += ((size_t)p.batch * p.seq * p.num_heads * p.head_size * 4 + 255) & ~(size_t)255;
  w.base = off;
  // prompts on the tensor-core kernel: the transposed value rows of every (batch, kv head)
  w.vt = off;
  if (p.seq > 1 && p.head_size == 128) off += (gqa_umma_vt_bytes(p.batch, p.kv_heads, p.cap) + 255) & ~(size_t)255;
  w.total = off;
  return w;
}

template <typename T, int EPL, int RP>
cudaError_t launch_decode_t(const GqaKP& kp, cudaStream_t st) {
  if constexpr (RP * EPL > 64) {
    return cudaErrorInvalidValue;  // never selected: decode_path() sends these to the generic path
  } else {
  const int D = EPL * 32;
  const int tile = kKT * D * (int)sizeof(T);
  int stages = tile <= 8192 ? 4 : tile <= 16384 ? 3 : 2;
  DecodeSmem L = decode_smem_layout(D, (int)sizeof(T), RP, stages);
  auto kern = gqa_decode_kernel<T, EPL, RP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total);
  if (e != cudaSuccess) return e;
  dim3 grid(kp.splits, kp.HK, kp.B);
  return launch_k(kern, grid, dim3((kNW + 1) * 32), (size_t)L.total, st, kp, stages);
  }
}

template <typename T, int EPL>
cudaError_t launch_decode_rp(const GqaKP& kp, cudaStream_t st) {
  switch (pow2_at_least(kp.R)) {
    case 1: return launch_decode_t<T, EPL, 1>(kp, st);
    case 2: return launch_decode_t<T, EPL, 2>(kp, st);
    case 4: return launch_decode_t<T, EPL, 4>(kp, st);
    case 8: return launch_decode_t<T, EPL, 8>(kp, st);
    case 16: return launch_decode_t<T, EPL, 16>(kp, st);
    case 32: return launch_decode_t<T, EPL, 32>(kp, st);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
cudaError_t launch_decode(const GqaKP& kp, cudaStream_t st) {
  switch (kp.D) {
    case 32: return launch_decode_rp<T, 1>(kp, st);
    case 64: return launch_decode_rp<T, 2>(kp, st);
    case 96: return launch_decode_rp<T, 3>(kp, st);
    case 128: return launch_decode_rp<T, 4>(kp, st);
    case 256: return launch_decode_rp<T, 8>(kp, st);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
cudaError_t launch_generic(const GqaKP& kp, cudaStream_t st) {
  const int warps = 4;
  const int items = kp.B * kp.S * (kp.H + kp.HK);
  cudaError_t e = launch_k(gqa_append_kernel<T>, dim3(div_up(items, warps)), dim3(warps * 32),
                           warps * kp.D * sizeof(float), st, kp);
  if (e != cudaSuccess) return e;
  const size_t smem = (size_t)(kp.D + kp.cap + 4) * sizeof(float);
  auto kern = gqa_generic_kernel<T>;
  if (smem > 48 * 1024) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_k(kern, dim3(kp.B * kp.S * kp.H), dim3(128), smem, st, kp);
}


bool mma_decode_path(const b200ep_gqa_params& p, int dtype) {
  const int G = (int)(p.num_heads / p.kv_heads);
  return p.seq == 1 && (dtype == kF16 || dtype == kBF16) && (p.head_size == 64 || p.head_size == 128) &&
         G >= 1 && G <= 8 && !getenv("ONNXRUNTIME_EP_B200_GQA_SIMT");
}

// splits of one (batch, kv-head) = cluster size (at most 8, the portable limit): one 32-key unit
// per warp at full capacity where that fits — decode attention is latency-bound at short contexts
// — but no more than two waves of CTAs over the SMs need (one CTA per SM: 207 KB of shared
// memory), so that many sequences (batch x kv heads >= 148) stream longer runs per CTA.
int mma_splits(const b200ep_gqa_params& p) {
  // one wave: the kernel holds one CTA per SM (its K / V streams fill shared memory)
  const int64_t units = (p.cap + kUnit - 1) / kUnit;
  const int64_t heads = std::max<int64_t>(1, p.batch * p.kv_heads);
  const int64_t by_sms = std::max<int64_t>(1, num_sms() / heads);
  return (int)std::max<int64_t>(1, std::min<int64_t>({8, (units + kMmaWarps - 1) / kMmaWarps, by_sms}));
}

template <typename T, int D, bool PAGED = false>
cudaError_t launch_mma_decode(const GqaKP& kp, int splits, cudaStream_t st) {
  using L = MmaSmem<D>;
  auto kern = gqa_mma_decode_kernel<T, D, PAGED>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(splits, kp.HK, kp.B);
  cfg.blockDim = dim3(kMmaWarps * 32);
  cfg.dynamicSmemBytes = L::kTotal;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, kp);
}

// prompt rows (S > 1) beyond what the split-K decode kernel holds: tensor-core prefill
bool mma_prefill_path(const b200ep_gqa_params& p, int dtype, int esz) {
  return p.seq > 1 && (dtype == kF16 || dtype == kBF16) && (p.head_size == 64 || p.head_size == 128) &&
         p.bias_batch == 0 && !decode_path(p, esz) && !getenv("ONNXRUNTIME_EP_B200_GQA_SIMT");
}

template <typename T, int D>
cudaError_t launch_paged_prefill_t(const GqaKP& kp, int max_rows, cudaStream_t st) {
  auto kern = gqa_mma_prefill_kernel<T, D, true>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PfSmem<D>::kTotal);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return launch_k(kern, dim3(div_up(max_rows, kPfRows), kp.H, kp.p_batch), dim3(kPfWarps * 32),
                  (size_t)PfSmem<D>::kTotal, st, kp);
}

template <typename T, int D>
cudaError_t launch_mma_prefill(const GqaKP& kp, cudaStream_t st) {
  const int warps = 4;
  const int items = kp.B * kp.S * (kp.H + kp.HK);
  cudaError_t e = launch_k(gqa_append_kernel<T>, dim3(div_up(items, warps)), dim3(warps * 32),
                           warps * kp.D * sizeof(float), st, kp);
  if (e != cudaSuccess) return e;
  auto kern = gqa_mma_prefill_kernel<T, D>;
  static bool configured = false;
  if (!configured) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PfSmem<D>::kTotal);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return launch_k(kern, dim3(div_up(kp.S, kPfRows), kp.H, kp.B), dim3(kPfWarps * 32), (size_t)PfSmem<D>::kTotal,
                  st, kp);
}
}  // namespace

size_t gqa_workspace_bytes(const b200ep_gqa_params& p) { return ws_layout(p).total; }
size_t gqa_workspace_min_bytes(const b200ep_gqa_params& p) { return ws_layout(p).base; }

// PagedAttention prompt chunks on the tensor-core prefill kernel: the caller has appended the new
// k / v rows and written the rotated q rows into `out`.
cudaError_t launch_paged_prefill(const PagedMmaArgs& a, cudaStream_t st) {
  GqaKP kp{};
  kp.kv_k = a.key_cache;
  kp.kv_v = a.value_cache;
  kp.out = a.out;
  kp.err = device_error_slot();
  kp.B = a.batch;
  kp.S = a.num_tokens;
  kp.H = a.num_heads;
  kp.HK = a.kv_heads;
  kp.D = a.head_size;
  kp.G = a.num_heads / a.kv_heads;
  kp.max_seq = a.max_seq;
  kp.do_rotary = a.do_rotary ? 1 : 0;
  kp.scale_log2 = a.scale * kLog2e;
  kp.p_cum = a.cum;
  kp.p_past = a.past;
  kp.p_bt = a.block_table;
  kp.p_batch = a.batch;
  kp.p_nblocks = a.num_blocks;
  kp.p_bs = a.block_size;
  kp.p_maxb = a.max_blocks;
  // rows of the longest sequence are not known on the host: every sequence gets the row blocks
  // of all packed rows, and the CTAs past its own rows exit at once
  if (a.dtype == kF16)
    return a.head_size == 64 ? launch_paged_prefill_t<__half, 64>(kp, a.num_tokens, st)
                             : launch_paged_prefill_t<__half, 128>(kp, a.num_tokens, st);
  return a.head_size == 64 ? launch_paged_prefill_t<__nv_bfloat16, 64>(kp, a.num_tokens, st)
                           : launch_paged_prefill_t<__nv_bfloat16, 128>(kp, a.num_tokens, st);
}

// PagedAttention rows on the tensor-core decode kernel (the caller has appended the new rows).
cudaError_t launch_paged_mma(const PagedMmaArgs& a, cudaStream_t st) {
  GqaKP kp{};
  kp.q = a.query;
  kp.kv_k = a.key_cache;
  kp.kv_v = a.value_cache;
  kp.cos_c = a.cos_cache;
  kp.sin_c = a.sin_cache;
  kp.out = a.out;
  kp.err = device_error_slot();
  kp.B = a.num_tokens;
  kp.S = 1;
  kp.H = a.num_heads;
  kp.HK = a.kv_heads;
  kp.D = a.head_size;
  kp.G = a.num_heads / a.kv_heads;
  kp.R = kp.G;
  kp.max_seq = a.max_seq;
  kp.half = a.rotary_half;
  kp.do_rotary = a.do_rotary ? 1 : 0;
  kp.interleaved = a.interleaved ? 1 : 0;
  kp.qstride = (int64_t)a.num_heads * a.head_size;
  kp.scale_log2 = a.scale * kLog2e;
  kp.p_cum = a.cum;
  kp.p_past = a.past;
  kp.p_bt = a.block_table;
  kp.p_batch = a.batch;
  kp.p_nblocks = a.num_blocks;
  kp.p_bs = a.block_size;
  kp.p_maxb = a.max_blocks;
  // one wave: the kernel holds one CTA per SM (its K / V streams fill shared memory)
  const int64_t heads = std::max<int64_t>(1, (int64_t)a.num_tokens * a.kv_heads);
  const int splits = (int)std::max<int64_t>(1, std::min<int64_t>(8, num_sms() / heads));
  if (a.dtype == kF16)
    return a.head_size == 64 ? launch_mma_decode<__half, 64, true>(kp, splits, st)
                             : launch_mma_decode<__half, 128, true>(kp, splits, st);
  return a.head_size == 64 ? launch_mma_decode<__nv_bfloat16, 64, true>(kp, splits, st)
                           : launch_mma_decode<__nv_bfloat16, 128, true>(kp, splits, st);
}

int launch_gqa(const GqaArgs& a, cudaStream_t st) {
  const b200ep_gqa_params& p = a.p;
  B200EP_CHECK_ARG(p.batch > 0 && p.seq > 0 && p.num_heads > 0 && p.kv_heads > 0 && p.head_size > 0,
                   "GroupQueryAttention: batch, seq, num_heads, kv_heads and head_size must be > 0");
  B200EP_CHECK_ARG(p.num_heads % p.kv_heads == 0, "GroupQueryAttention: num_heads % kv_num_heads != 0");
  B200EP_CHECK_ARG(p.head_size <= 256, "GroupQueryAttention: head_size > 256 is not supported");
  B200EP_CHECK_ARG(p.cap > 0, "GroupQueryAttention: KV buffer capacity must be > 0");
  B200EP_CHECK_ARG(is_float_dtype(a.dtype), "GroupQueryAttention: dtype must be float32/float16/bfloat16");
  B200EP_CHECK_ARG(a.query && a.kv_key && a.kv_value && a.seqlens_k && a.out,
                   "GroupQueryAttention: null tensor pointer");
  B200EP_CHECK_ARG(p.packed_qkv || (a.key && a.value), "GroupQueryAttention: key/value missing");
  if (p.do_rotary) {
    B200EP_CHECK_ARG(a.cos_cache && a.sin_cache && p.rotary_half > 0 && 2 * p.rotary_half <= p.head_size &&
                         p.max_seq > 0,
                     "GroupQueryAttention: do_rotary needs cos/sin caches with 2*rotary_half <= head_size");
    B200EP_CHECK_ARG(p.rotary_half <= 128, "GroupQueryAttention: rotary_half > 128 is not supported");
  }
  B200EP_CHECK_ARG((a.q_norm == nullptr) == (a.k_norm == nullptr),
                   "GroupQueryAttention: q_norm and k_norm must be given together");
  B200EP_CHECK_ARG(p.bias_batch == 0 || a.bias, "GroupQueryAttention: attention_bias pointer missing");
  const int esz = dtype_size(a.dtype);
  const WsLayout wl = ws_layout(p);
  B200EP_CHECK_ARG(a.workspace && a.workspace_bytes >= wl.base, "GroupQueryAttention: workspace too small");

  GqaKP kp{};
  kp.q = a.query;
  kp.k = p.packed_qkv ? a.query : a.key;
  kp.v = p.packed_qkv ? a.query : a.value;
  kp.kv_k = a.kv_key;
  kp.kv_v = a.kv_value;
  kp.seqlens = a.seqlens_k;
  kp.cos_c = a.cos_cache;
  kp.sin_c = a.sin_cache;
  kp.qn = a.q_norm;
  kp.kn = a.k_norm;
  kp.bias = p.bias_batch > 0 ? a.bias : nullptr;
  kp.out = a.out;
  char* ws = static_cast<char*>(a.workspace);
  kp.counters = reinterpret_cast<int*>(ws + wl.counters);
  kp.partial = reinterpret_cast<float*>(ws + wl.partial);
  kp.qrot = reinterpret_cast<float*>(ws + wl.qrot);
  kp.err = device_error_slot();
  kp.B = (int)p.batch;
  kp.S = (int)p.seq;
  kp.H = (int)p.num_heads;
  kp.HK = (int)p.kv_heads;
  kp.D = (int)p.head_size;
  kp.G = kp.H / kp.HK;
  kp.R = kp.S * kp.G;
  kp.cap = (int)p.cap;
  kp.max_seq = (int)p.max_seq;
  kp.half = (int)p.rotary_half;
  kp.splits = choose_splits(p);
  kp.do_rotary = p.do_rotary ? 1 : 0;
  kp.interleaved = p.interleaved ? 1 : 0;
  kp.local_window = p.local_window;
  const int64_t D = p.head_size;
  kp.qstride = p.packed_qkv ? (p.num_heads + 2 * p.kv_heads) * D : p.num_heads * D;
  kp.kstride = p.packed_qkv ? kp.qstride : p.kv_heads * D;
  kp.koff = p.packed_qkv ? p.num_heads * D : 0;
  kp.voff = p.packed_qkv ? (p.num_heads + p.kv_heads) * D : 0;
  kp.bias_batch = (int)p.bias_batch;
  kp.bias_total = (int)p.bias_total;
  const float scale = p.scale != 0.f ? p.scale : 1.0f / sqrtf((float)D);
  kp.scale_log2 = scale * kLog2e;
  kp.qk_eps = p.qk_norm_eps;
  kp.has_qk_norm = a.q_norm ? 1 : 0;

  const bool aligned = (reinterpret_cast<uintptr_t>(a.kv_key) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(a.kv_value) % 16 == 0);
  cudaError_t e;
  if (mma_decode_path(p, a.dtype) && aligned) {
    const int sp = mma_splits(p);
    if (a.dtype == kF16)
      e = p.head_size == 64 ? launch_mma_decode<__half, 64>(kp, sp, st) : launch_mma_decode<__half, 128>(kp, sp, st);
    else
      e = p.head_size == 64 ? launch_mma_decode<__nv_bfloat16, 64>(kp, sp, st)
                            : launch_mma_decode<__nv_bfloat16, 128>(kp, sp, st);
  } else if (mma_prefill_path(p, a.dtype, esz) && aligned && a.workspace_bytes >= wl.total &&
             gqa_umma_supported(p.batch, p.kv_heads, p.head_size, p.cap, a.dtype)) {
    // tcgen05 prompt kernel: append (rotate q into the workspace, k / v into the cache), then it
    const int warps = 4;
    const int items = kp.B * kp.S * (kp.H + kp.HK);
    e = launch_k(a.dtype == kF16 ? gqa_append_kernel<__half> : gqa_append_kernel<__nv_bfloat16>,
                 dim3(div_up(items, warps)), dim3(warps * 32), warps * kp.D * sizeof(float), st, kp);
    if (e == cudaSuccess) {
      UmmaAttnArgs u{};
      u.qrot = kp.qrot;
      u.kv_k = a.kv_key;
      u.kv_v = a.kv_value;
      u.vt = ws + wl.vt;
      u.seqlens = a.seqlens_k;
      u.out = a.out;
      u.err = kp.err;
      u.B = kp.B, u.S = kp.S, u.H = kp.H, u.HK = kp.HK, u.G = kp.G, u.cap = kp.cap, u.max_seq = kp.max_seq;
      u.do_rotary = kp.do_rotary, u.local_window = kp.local_window, u.lt = (int)gqa_umma_lt(p.cap);
      u.dtype = a.dtype;
      u.scale_log2 = kp.scale_log2;
      e = launch_gqa_umma_prefill(u, st);
    }
  } else if (mma_prefill_path(p, a.dtype, esz) && aligned) {
    if (a.dtype == kF16)
      e = p.head_size == 64 ? launch_mma_prefill<__half, 64>(kp, st) : launch_mma_prefill<__half, 128>(kp, st);
    else
      e = p.head_size == 64 ? launch_mma_prefill<__nv_bfloat16, 64>(kp, st)
                            : launch_mma_prefill<__nv_bfloat16, 128>(kp, st);
  } else if (decode_path(p, esz) && aligned) {
    switch (a.dtype) {
      case kF32: e = launch_decode<float>(kp, st); break;
      case kF16: e = launch_decode<__half>(kp, st); break;
      default: e = launch_decode<__nv_bfloat16>(kp, st); break;
    }
  } else {
    B200EP_CHECK_ARG(p.cap <= 40000, "GroupQueryAttention: generic path limited to cap <= 40000");
    switch (a.dtype) {
      case kF32: e = launch_generic<float>(kp, st); break;
      case kF16: e = launch_generic<__half>(kp, st); break;
      default: e = launch_generic<__nv_bfloat16>(kp, st); break;
    }
  }
  return cuda_status(e, "GroupQueryAttention launch");
}

}  // namespace b200ep
