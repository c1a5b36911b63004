// PagedAttention for sm_100a (reference: paged_attention_op, rust/src/ops/attention.rs:2495-2746,
// which gathers the cached prefix through the block table with mlx_take, scatters the new rows
// with mlx_scatter and runs a masked SDPA per sequence).
//
// Two launches, both reading the control tensors (cumulative lengths, past lengths, block table)
// on the device, so nothing is copied to the host.  Rows with head_size 64 / 128 and at most 8
// query heads per kv head attend on the tensor-core decode kernel of gqa.cu
// (gqa_mma_decode_kernel<..., PAGED = true>: per-warp cp.async K / V streams whose row addresses
// go through the block table, mma.sync scores, cluster merge), or, for prompt chunks (16 rows or
// more per sequence on average), on its prefill kernel (gqa_mma_prefill_kernel<..., PAGED = true>:
// 64-row query tiles against 64-key tiles fetched through the block table, the rotated q rows
// handed over in the output buffer); paged_attn_kernel covers the rest.
//   paged_append_kernel — one CTA per packed token: finds its sequence, RoPEs the new k row at
//     position past_b + j (fp32, rounded once to the I/O dtype) and writes k and v into their
//     block-table slot of the caches.
//   paged_attn_kernel   — a thread-block cluster of up to 8 CTAs per (token, kv head, chunk of
//     1 / 2 / 4 / 8 query heads), 8 warps each; the cluster splits the causal key range
//     [0, past_b + j] into 32-key chunks.  Every CTA RoPEs its query rows into shared memory
//     (rounded through the I/O dtype, then scaled); each warp takes chunks in turn: lane l
//     scores key 32c + l against every query row (16-byte loads of the key row through the
//     block table), an fp32 online softmax runs per warp, and P.V accumulates with lanes owning
//     head_size / 32 dims of each value row (coalesced, 8 rows in flight).  Warp states merge in
//     shared memory, the cluster's CTA states in rank 0 through distributed shared memory.
// A slot outside the caches / block table, or a position outside the cos / sin rows, is never
// read or written: the append skips it, attention masks the key (the tensor-core path reads it as
// zeros; a query row whose own position is out of range is left unwritten there and zeroed here),
// and the device error word records it.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <string>

#include "common.cuh"
#include "kernels/kernels.h"

namespace b200ep {

DeviceErrorSlot* device_error_slot();

namespace {

enum { kErrPagedSlot = 121 };
constexpr int kPagedWarps = 8;   // warps per attention CTA
constexpr int kPagedGroup = 8;   // query heads per attention CTA

struct PagedKP {
  const void* q;
  const void* k;
  const void* v;
  void* kc;
  void* vc;
  const int32_t* cum;
  const int32_t* past;
  const int32_t* bt;
  const void* cos_c;
  const void* sin_c;
  void* out;
  DeviceErrorSlot* err;
  int batch, ntok, H, HK, D, G, gm, gchunks, nblocks, bs, maxb, max_seq, half, rot, inter;
  int qout;  // the append also writes the rotated q rows (rounded) into out (prompt path)
  float scale;
};

// The sequence owning packed row i: the b with cum[b] <= i < cum[b + 1], or -1.
__device__ int seq_of(const PagedKP& kp, int i) {
  int lo = 0, hi = kp.batch;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(kp.cum + mid) <= i) lo = mid;
    else hi = mid - 1;
  }
  if (lo >= kp.batch || __ldg(kp.cum + lo) > i || i >= __ldg(kp.cum + lo + 1)) return -1;
  return lo;
}

// Cache row (physical block * block_size + offset) of position pos of sequence b, or -1.
__device__ int slot_of(const PagedKP& kp, int b, int pos) {
  if (pos < 0) return -1;
  const int blk = pos / kp.bs;
  if (blk >= kp.maxb) return -1;
  const int phys = __ldg(kp.bt + (size_t)b * kp.maxb + blk);
  if (phys < 0 || phys >= kp.nblocks) return -1;
  return phys * kp.bs + pos % kp.bs;
}

// Element i of head vector x (fp32) after RoPE at position pos (attention.rs:417-461 forms):
// halves (i, i + half) or interleaved pairs (2i, 2i + 1); dims past 2 * half pass through.
template <typename T>
__device__ float rope_at(const float* x, int i, const PagedKP& kp, int pos) {
  if (!kp.rot || i >= 2 * kp.half) return x[i];
  int pi;
  bool first;
  float a, b;
  if (!kp.inter) {
    first = i < kp.half;
    pi = first ? i : i - kp.half;
    a = x[pi], b = x[pi + kp.half];
  } else {
    first = !(i & 1);
    pi = i >> 1;
    a = x[2 * pi], b = x[2 * pi + 1];
  }
  const float c = to_f<T>(static_cast<const T*>(kp.cos_c)[(size_t)pos * kp.half + pi]);
  const float s = to_f<T>(static_cast<const T*>(kp.sin_c)[(size_t)pos * kp.half + pi]);
  return first ? __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s)) : __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
}

template <typename T>
__global__ void __launch_bounds__(128) paged_append_kernel(PagedKP kp) {
  extern __shared__ float xs[];  // [max(heads, kv_heads) * head_size] one row, fp32
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x;
  const int b = seq_of(kp, i);
  const int pos = b >= 0 ? __ldg(kp.past + b) + (i - __ldg(kp.cum + b)) : -1;
  const bool pos_ok = pos >= 0 && !(kp.rot && pos >= kp.max_seq);
  const int slot = pos_ok ? slot_of(kp, b, pos) : -1;
  if (slot < 0 && threadIdx.x == 0) report_device_error(kp.err, kErrPagedSlot, i);
  if (!pos_ok) return;
  if (slot >= 0) {
    const int row = kp.HK * kp.D;
    const T* K = static_cast<const T*>(kp.k) + (size_t)i * row;
    const T* V = static_cast<const T*>(kp.v) + (size_t)i * row;
    for (int e = threadIdx.x; e < row; e += blockDim.x) xs[e] = to_f<T>(K[e]);
    __syncthreads();
    T* kc = static_cast<T*>(kp.kc) + (size_t)slot * row;
    T* vc = static_cast<T*>(kp.vc) + (size_t)slot * row;
    for (int e = threadIdx.x; e < row; e += blockDim.x) {
      const int h = e / kp.D;
      kc[e] = from_f<T>(rope_at<T>(xs + h * kp.D, e - h * kp.D, kp, pos));
      vc[e] = V[e];
    }
  }
  if (kp.qout) {  // the prompt kernel reads the rotated q rows from out
    __syncthreads();
    const int row = kp.H * kp.D;
    const T* Q = static_cast<const T*>(kp.q) + (size_t)i * row;
    for (int e = threadIdx.x; e < row; e += blockDim.x) xs[e] = to_f<T>(Q[e]);
    __syncthreads();
    T* O = static_cast<T*>(kp.out) + (size_t)i * row;
    for (int e = threadIdx.x; e < row; e += blockDim.x) {
      const int h = e / kp.D;
      O[e] = from_f<T>(rope_at<T>(xs + h * kp.D, e - h * kp.D, kp, pos));
    }
  }
}

template <typename T>
__device__ __forceinline__ void unpack8f(uint4 w, float (&f)[8]) {
  const T* h = reinterpret_cast<const T*>(&w);
#pragma unroll
  for (int u = 0; u < 8; ++u) f[u] = to_f<T>(h[u]);
}

template <typename T, int DPL, int GM>
__global__ void __launch_bounds__(kPagedWarps * 32, 2) paged_attn_kernel(PagedKP kp) {
  constexpr int D = DPL * 32, NW = kPagedWarps;
  __shared__ __align__(16) float qs[GM][D];  // rotated, rounded, scaled query rows
  __shared__ float wm[NW][GM], wl[NW][GM];
  __shared__ __align__(16) float wo[NW][GM][D];  // per-warp P.V (and the raw q rows first)
  __shared__ __align__(16) float cs[GM][D + 2];  // this CTA's merged (o, m, l), read by cluster rank 0
  pdl_wait();
  pdl_trigger();
  uint32_t crank, csize;
  asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
  asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(csize));
  const int i = blockIdx.x / csize;  // packed token; the cluster splits its keys
  const int hk = blockIdx.y / kp.gchunks, g0 = (blockIdx.y % kp.gchunks) * GM;
  const int ng = min(GM, kp.G - g0);
  const int hq0 = hk * kp.G + g0;  // first query head of this CTA
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  T* out = static_cast<T*>(kp.out) + (size_t)i * kp.H * D + (size_t)hq0 * D;

  const int b = seq_of(kp, i);
  const int pos = b >= 0 ? __ldg(kp.past + b) + (i - __ldg(kp.cum + b)) : -1;
  const bool valid = pos >= 0 && !(kp.rot && pos >= kp.max_seq);  // the same in every CTA of the cluster
  if (valid) {
    // query rows: raw into wo[0], then rotated / rounded / scaled into qs
    float* raw = &wo[0][0][0];
    const T* Q = static_cast<const T*>(kp.q) + (size_t)i * kp.H * D + (size_t)hq0 * D;
    for (int e = threadIdx.x; e < ng * D; e += blockDim.x) raw[e] = to_f<T>(Q[e]);
    __syncthreads();
    for (int e = threadIdx.x; e < GM * D; e += blockDim.x) {
      const int g = e / D, d = e - g * D;
      qs[g][d] = g < ng ? round_through<T>(rope_at<T>(raw + g * D, d, kp, pos)) * kp.scale : 0.f;
    }
    __syncthreads();
  }

  const int row = kp.HK * D;
  const T* KC = static_cast<const T*>(kp.kc) + (size_t)hk * D;
  const T* VC = static_cast<const T*>(kp.vc) + (size_t)hk * D;
  const int n = valid ? pos + 1 : 0;  // causal: keys 0 .. pos
  const int nch = (n + 31) / 32;       // 32-key chunks, split evenly over the cluster
  const int cbeg = (int)((int64_t)nch * crank / csize), cend = (int)((int64_t)nch * (crank + 1) / csize);
  float m[GM], l[GM], acc[GM][DPL];
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    m[g] = -INFINITY, l[g] = 0.f;
#pragma unroll
    for (int d = 0; d < DPL; ++d) acc[g][d] = 0.f;
  }
  bool bad = false;
  for (int c = cbeg + warp; c < cend; c += NW) {
    const int kk = c * 32 + lane;
    const int slot = kk < n ? slot_of(kp, b, kk) : -1;
    bad |= kk < n && slot < 0;
    float s[GM];
#pragma unroll
    for (int g = 0; g < GM; ++g) s[g] = slot >= 0 ? 0.f : -INFINITY;
    if (slot >= 0) {
      const uint4* kr = reinterpret_cast<const uint4*>(KC + (size_t)slot * row);
#pragma unroll
      for (int u0 = 0; u0 < D / 8; u0 += 8) {
        uint4 w[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (u0 + u < D / 8) w[u] = __ldg(kr + u0 + u);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (u0 + u >= D / 8) break;
          float kf[8];
          unpack8f<T>(w[u], kf);
#pragma unroll
          for (int g = 0; g < GM; ++g) {
            const float4 qa = *reinterpret_cast<const float4*>(&qs[g][(u0 + u) * 8]);
            const float4 qb = *reinterpret_cast<const float4*>(&qs[g][(u0 + u) * 8 + 4]);
            s[g] += qa.x * kf[0] + qa.y * kf[1] + qa.z * kf[2] + qa.w * kf[3] + qb.x * kf[4] + qb.y * kf[5] +
                    qb.z * kf[6] + qb.w * kf[7];
          }
        }
      }
    }
    // fp32 online softmax per query row (warp-uniform max; masked keys contribute 0)
    float p[GM];
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      const float mn = fmaxf(m[g], warp_max(s[g]));
      const float alpha = m[g] == -INFINITY ? 0.f : __expf(m[g] - mn);
      p[g] = s[g] == -INFINITY ? 0.f : __expf(s[g] - mn);
      l[g] = l[g] * alpha + p[g];
      m[g] = mn;
#pragma unroll
      for (int d = 0; d < DPL; ++d) acc[g][d] *= alpha;
    }
    // P.V: lanes own dims [lane * DPL, lane * DPL + DPL) of each value row; 8 rows in flight
    const int nk = min(32, n - c * 32);
    for (int t0 = 0; t0 < nk; t0 += 8) {
      int st[8];
      float vf[8][DPL];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        st[u] = __shfl_sync(0xffffffffu, slot, t0 + u);  // -1 past the chunk's keys
        const T* vr = VC + (size_t)(st[u] < 0 ? 0 : st[u]) * row + lane * DPL;
        if constexpr (DPL == 4) {
          uint2 w = make_uint2(0, 0);
          if (st[u] >= 0) w = __ldg(reinterpret_cast<const uint2*>(vr));
          const T* h = reinterpret_cast<const T*>(&w);
#pragma unroll
          for (int d = 0; d < 4; ++d) vf[u][d] = to_f<T>(h[d]);
        } else if constexpr (DPL == 2) {
          uint32_t w = 0;
          if (st[u] >= 0) w = __ldg(reinterpret_cast<const uint32_t*>(vr));
          const T* h = reinterpret_cast<const T*>(&w);
          vf[u][0] = to_f<T>(h[0]), vf[u][1] = to_f<T>(h[1]);
        } else {
          vf[u][0] = st[u] >= 0 ? to_f<T>(vr[0]) : 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int g = 0; g < GM; ++g) {
          const float pt = __shfl_sync(0xffffffffu, p[g], t0 + u);  // 0 for masked / absent keys
#pragma unroll
          for (int d = 0; d < DPL; ++d) acc[g][d] = fmaf(pt, vf[u][d], acc[g][d]);
        }
    }
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) report_device_error(kp.err, kErrPagedSlot, i);
  __syncthreads();  // raw (wo[0]) is no longer read
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    const float lw = warp_sum(l[g]);
    if (lane == 0) wm[warp][g] = m[g], wl[warp][g] = lw;
#pragma unroll
    for (int d = 0; d < DPL; ++d) wo[warp][g][lane * DPL + d] = acc[g][d];
  }
  __syncthreads();
  // this CTA's state: o and l relative to its own max m
  for (int e = threadIdx.x; e < GM * D; e += blockDim.x) {
    const int g = e / D, d = e - g * D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) mx = fmaxf(mx, wm[w][g]);
    float den = 0.f, num = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      if (wm[w][g] == -INFINITY) continue;
      const float f = __expf(wm[w][g] - mx);
      den += wl[w][g] * f;
      num += wo[w][g][d] * f;
    }
    cs[g][d] = num;
    if (d == 0) cs[g][D] = mx, cs[g][D + 1] = den;
  }
  // rank 0 combines the cluster's states through distributed shared memory; the second barrier
  // keeps every CTA's shared memory alive until rank 0 has read it
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (crank == 0) {
    for (int e = threadIdx.x; e < ng * D; e += blockDim.x) {
      const int g = e / D, d = e - g * D;
      const uint32_t base = smem_u32(&cs[g][0]);
      float mx = -INFINITY, den = 0.f, num = 0.f;  // running merge in rank order
      for (uint32_t r = 0; r < csize; ++r) {
        uint32_t ra;
        float orr, mr, lr;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(base), "r"(r));
        asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(orr) : "r"(ra + (uint32_t)(d * 4)));
        asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(mr) : "r"(ra + (uint32_t)(D * 4)));
        asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(lr) : "r"(ra + (uint32_t)((D + 1) * 4)));
        if (mr == -INFINITY) continue;
        const float mn = fmaxf(mx, mr);
        const float a = mx == -INFINITY ? 0.f : __expf(mx - mn), f = __expf(mr - mn);
        den = den * a + lr * f;
        num = num * a + orr * f;
        mx = mn;
      }
      out[e] = from_f<T>(den > 0.f ? num / den : 0.f);
    }
    if (!valid && threadIdx.x == 0) report_device_error(kp.err, kErrPagedSlot, i);
  }
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <typename T, int DPL, int GM>
cudaError_t launch_attn(const PagedKP& kp, int splits, cudaStream_t st) {
  auto kern = paged_attn_kernel<T, DPL, GM>;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(kp.ntok * splits), (unsigned)(kp.HK * kp.gchunks));
  cfg.blockDim = dim3(kPagedWarps * 32);
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

template <typename T, int DPL>
cudaError_t launch_attn_g(const PagedKP& kp, int splits, cudaStream_t st) {
  switch (kp.gm) {
    case 1: return launch_attn<T, DPL, 1>(kp, splits, st);
    case 2: return launch_attn<T, DPL, 2>(kp, splits, st);
    case 4: return launch_attn<T, DPL, 4>(kp, splits, st);
  }
  return launch_attn<T, DPL, 8>(kp, splits, st);
}

template <typename T>
cudaError_t launch_paged_t(const PagedKP& kp_in, int dtype, cudaStream_t st) {
  PagedKP kp = kp_in;
  const bool mma = (kp.D == 64 || kp.D == 128) && kp.G <= 8 && kp.ntok < 65536 &&
                   reinterpret_cast<uintptr_t>(kp.q) % 8 == 0 && !getenv("ONNXRUNTIME_EP_B200_PAGED_SIMT");
  // prompt chunks (16 rows or more per sequence on average) attend as 64-row tiles on the
  // tensor-core prefill kernel of gqa.cu, which reads the rotated q rows the append leaves in out
  const bool prompt = mma && (int64_t)kp.ntok >= 16ll * kp.batch && kp.batch <= 65535 &&
                      (size_t)kp.H * kp.D * sizeof(float) <= 48 * 1024 &&
                      reinterpret_cast<uintptr_t>(kp.out) % 4 == 0;
  kp.qout = prompt ? 1 : 0;
  const size_t app_smem = (size_t)(prompt ? std::max(kp.H, kp.HK) : kp.HK) * kp.D * sizeof(float);
  if (app_smem > 48 * 1024) return cudaErrorInvalidValue;
  if (cudaError_t e = launch_k(paged_append_kernel<T>, dim3((unsigned)kp.ntok), dim3(128), app_smem, st, kp))
    return e;
  // the tensor-core decode kernel of gqa.cu (cp.async K / V streams, mma.sync scores) where it
  // applies; the SIMT kernel below otherwise
  if (mma) {
    PagedMmaArgs a{};
    a.query = kp.q, a.key_cache = kp.kc, a.value_cache = kp.vc;
    a.cum = kp.cum, a.past = kp.past, a.block_table = kp.bt;
    a.cos_cache = kp.cos_c, a.sin_cache = kp.sin_c, a.out = kp.out;
    a.dtype = dtype, a.batch = kp.batch, a.num_tokens = kp.ntok, a.num_heads = kp.H, a.kv_heads = kp.HK;
    a.head_size = kp.D, a.num_blocks = kp.nblocks, a.block_size = kp.bs, a.max_blocks = kp.maxb;
    a.max_seq = kp.max_seq, a.rotary_half = kp.half, a.do_rotary = kp.rot, a.interleaved = kp.inter;
    a.scale = kp.scale;
    return prompt ? launch_paged_prefill(a, st) : launch_paged_mma(a, st);
  }
  // key splits per (token, kv head, query-head chunk): as many as fit one wave of the two CTAs
  // per SM (a partial second wave would double the time of its keys), at most a portable cluster
  // of 8
  const int64_t items = (int64_t)kp.ntok * kp.HK * kp.gchunks;
  const int splits = (int)std::max<int64_t>(1, std::min<int64_t>(8, 2 * num_sms() / items));
  switch (kp.D) {
    case 32: return launch_attn_g<T, 1>(kp, splits, st);
    case 64: return launch_attn_g<T, 2>(kp, splits, st);
    case 128: return launch_attn_g<T, 4>(kp, splits, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace
}  // namespace b200ep

using namespace b200ep;

extern "C" B200EP_API int b200ep_paged_attention(const b200ep_paged_params* p, const void* query, const void* key,
                                                 const void* value, void* key_cache, void* value_cache,
                                                 const int32_t* cumulative_seqlens, const int32_t* past_seqlens,
                                                 const int32_t* block_table, const void* cos_cache,
                                                 const void* sin_cache, void* out, int dtype, void* stream) {
  try {
    B200EP_CHECK_ARG(p != nullptr, "PagedAttention: params is null");
    B200EP_CHECK_ARG(dtype == kF16 || dtype == kBF16, "PagedAttention: dtype must be float16 or bfloat16");
    B200EP_CHECK_ARG(p->batch > 0 && p->num_tokens >= 0 && p->num_heads > 0 && p->kv_heads > 0 &&
                         p->num_heads % p->kv_heads == 0,
                     "PagedAttention: batch > 0 and num_heads a positive multiple of kv_heads required");
    B200EP_CHECK_ARG(p->head_size == 32 || p->head_size == 64 || p->head_size == 128,
                     "PagedAttention: head_size must be 32, 64 or 128");
    B200EP_CHECK_ARG(p->num_blocks > 0 && p->block_size > 0 && p->max_blocks > 0 &&
                         (int64_t)p->num_blocks * p->block_size < (1ll << 31),
                     "PagedAttention: bad cache / block-table geometry");
    B200EP_CHECK_ARG(!p->do_rotary || (cos_cache && sin_cache && p->rotary_half > 0 &&
                                       2 * p->rotary_half <= p->head_size && p->max_seq > 0),
                     "PagedAttention: do_rotary needs cos/sin caches of [max_seq, rotary_half <= head_size / 2]");
    if (p->num_tokens == 0) return B200EP_OK;
    B200EP_CHECK_ARG(query && key && value && key_cache && value_cache && cumulative_seqlens && past_seqlens &&
                         block_table && out,
                     "PagedAttention: null pointer");
    B200EP_CHECK_ARG((reinterpret_cast<uintptr_t>(key_cache) | reinterpret_cast<uintptr_t>(value_cache)) % 16 == 0,
                     "PagedAttention: key / value caches must be 16-byte aligned");
    PagedKP kp{};
    kp.q = query, kp.k = key, kp.v = value, kp.kc = key_cache, kp.vc = value_cache;
    kp.cum = cumulative_seqlens, kp.past = past_seqlens, kp.bt = block_table;
    kp.cos_c = cos_cache, kp.sin_c = sin_cache, kp.out = out, kp.err = device_error_slot();
    kp.batch = p->batch, kp.ntok = p->num_tokens, kp.H = p->num_heads, kp.HK = p->kv_heads, kp.D = p->head_size;
    kp.G = p->num_heads / p->kv_heads;
    kp.gm = kp.G >= kPagedGroup ? kPagedGroup : kp.G > 2 ? 4 : kp.G;  // query heads per CTA (1, 2, 4 or 8)
    kp.gchunks = (kp.G + kp.gm - 1) / kp.gm;
    kp.nblocks = p->num_blocks, kp.bs = p->block_size, kp.maxb = p->max_blocks;
    kp.max_seq = p->max_seq, kp.half = p->rotary_half, kp.rot = p->do_rotary ? 1 : 0, kp.inter = p->interleaved ? 1 : 0;
    kp.scale = p->scale != 0.f ? p->scale : 1.f / std::sqrt((float)p->head_size);
    B200EP_CHECK_ARG((int64_t)kp.HK * kp.gchunks <= 65535 && (int64_t)kp.ntok * 8 < (1ll << 31),
                     "PagedAttention: too many kv heads or tokens");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const cudaError_t e =
        dtype == kF16 ? launch_paged_t<__half>(kp, dtype, st) : launch_paged_t<__nv_bfloat16>(kp, dtype, st);
    return cuda_status(e, "PagedAttention launch");
  } catch (const std::exception& e) {
    return set_error(B200EP_EINTERNAL, std::string("exception: ") + e.what());
  }
}
