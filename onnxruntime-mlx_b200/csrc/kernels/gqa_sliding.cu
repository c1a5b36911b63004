// GroupQueryAttention over a sliding-window KV cache (sliding_window_cache = 1, local_window_size =
// W; reference: the sliding branch of group_query_attention_op, rust/src/ops/attention.rs:725-880,
// claim 1552-1575).
//
// The cache holds at most `cap` (>= W) rows per (sequence, kv head).  After L tokens the resident
// rows are the last end(L) = L - gap * ceil((L - cap) / gap) of them once L exceeds cap (gap =
// cap - W + 1): rows are reclaimed from the front `gap` at a time.  For a step of S new rows of
// sequence b, p = seqlens_k[b] + 1 - S is the first new row's absolute position, before = end(p),
// after = end(p + S), kept = after - S rows of the past survive and seed_offset = before - kept are
// dropped.  The attention runs over `work` = past rows [seed_start, before) followed by the new rows
// (seed_start = seed_offset, or 0 in the staging form: when any sequence keeps fewer rows than its
// window needs, min(p, W - 1)), query i at work row seed_rows + i seeing work rows
// (seed_rows + i - W, seed_rows + i]; q and k are rotated at their absolute positions p + i.
// Present rows [0, after) are work rows [write_start, write_start + after) (write_start =
// seed_offset in the staging form, else 0), the rest of the capacity zero.
//
// Device work, in order on the caller's stream (every length is read on the device, so one launch
// sequence — and a CUDA graph holding it — serves every step):
//   1. sliding_geometry_kernel: per-sequence geometry and the staging decision (one CTA);
//   2. sliding_seed_kernel: the seed rows of past K / V into the work buffers;
//   3. sliding_rows_kernel: q and k rotated at their absolute positions (rounded to the I/O dtype,
//      as the other GQA paths store rotated rows) and v, into contiguous staging rows;
//   4. the GQA kernels of gqa.cu over the work buffers (no rotary, causal window W): they append the
//      new k / v rows at work rows [seed_rows, seed_rows + S) and write the attention output;
//   5. sliding_writeback_kernel: present = the kept work rows from row 0, zeros after them (present
//      may be the past buffers themselves: the work copy was taken first).
#include <algorithm>

#include "../common.cuh"
#include "kernels.h"

namespace b200ep {

namespace {

template <typename F>
cudaError_t by_float_dtype(int dt, F&& f) {
  switch (dt) {
    case kF32: return f(float{});
    case kF16: return f(__half{});
    case kBF16: return f(__nv_bfloat16{});
  }
  return cudaErrorInvalidValue;
}

struct SlidingGeo {
  int p, before, after, seed_start, write_start, seed_rows;
};

__device__ __forceinline__ int sliding_end(int len, int cap, int gap) {
  return len <= cap ? len : len - gap * ((len - cap + gap - 1) / gap);
}

enum { kErrSlidingPos = 211 };

__global__ void sliding_geometry_kernel(const int32_t* __restrict__ seqlens, int B, int S, int cap, int W,
                                        SlidingGeo* __restrict__ geo, int32_t* __restrict__ seq_w) {
  pdl_wait();
  pdl_trigger();
  const int gap = cap - W + 1;
  bool need = false;
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int p = max(seqlens[b] + 1 - S, 0);
    const int before = sliding_end(p, cap, gap), after = sliding_end(p + S, cap, gap);
    const int kept = after - S;
    need |= kept < min(p, W - 1);
    geo[b] = SlidingGeo{p, before, after, before - kept, 0, 0};
  }
  const bool staging = __syncthreads_or(need);
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    SlidingGeo g = geo[b];
    const int off = g.seed_start;  // seed_offset
    g.seed_start = staging ? 0 : off;
    g.write_start = staging ? off : 0;
    g.seed_rows = g.before - g.seed_start;
    geo[b] = g;
    seq_w[b] = g.seed_rows + S - 1;
  }
}

// rows [seed_start, before) of past -> rows [0, seed_rows) of work; grid (row blocks, HK, B), one
// 16-byte chunk per thread
template <typename T>
__global__ void sliding_seed_kernel(const T* __restrict__ pk, const T* __restrict__ pv, T* __restrict__ wk,
                                    T* __restrict__ wv, const SlidingGeo* __restrict__ geo, int HK, int cap,
                                    int wcap, int D) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.z, h = blockIdx.y;
  const SlidingGeo g = geo[b];
  const int cpr = D * (int)sizeof(T) / 16;  // 16-byte chunks per row
  const size_t src0 = ((size_t)b * HK + h) * cap * D, dst0 = ((size_t)b * HK + h) * wcap * D;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < g.seed_rows * cpr; i += gridDim.x * blockDim.x) {
    const int r = i / cpr, c = i - r * cpr;
    const size_t so = (src0 + (size_t)(g.seed_start + r) * D) * sizeof(T) + c * 16;
    const size_t dof = (dst0 + (size_t)r * D) * sizeof(T) + c * 16;
    *reinterpret_cast<uint4*>(reinterpret_cast<char*>(wk) + dof) =
        *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(pk) + so);
    *reinterpret_cast<uint4*>(reinterpret_cast<char*>(wv) + dof) =
        *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(pv) + so);
  }
}

// q / k rows rotated at absolute positions p + s and v rows, into contiguous [B, S, heads * D]
// staging rows; grid (S, B), threads over the (H + HK) heads' rotary pairs and v elements.  Inputs
// may be packed (q | k | v per row, width (H + 2 HK) D).
template <typename T>
__global__ void sliding_rows_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                                    int packed, T* __restrict__ qr, T* __restrict__ kr, T* __restrict__ vr,
                                    const T* __restrict__ cos_c, const T* __restrict__ sin_c,
                                    const SlidingGeo* __restrict__ geo, int S, int H, int HK, int D, int half,
                                    int interleaved, int do_rotary, int max_seq, DeviceErrorSlot* err) {
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.x, b = blockIdx.y;
  const int pos = geo[b].p + s;
  const bool rot = do_rotary && pos < max_seq;
  if (do_rotary && pos >= max_seq && threadIdx.x == 0) report_device_error(err, kErrSlidingPos, b);
  const size_t row = (size_t)b * S + s;
  const int wq = packed ? (H + 2 * HK) * D : H * D, wkv = packed ? wq : HK * D;
  const T* qrow = q + row * wq;
  const T* krow = (packed ? q : k) + row * wkv + (packed ? H * D : 0);
  const T* vrow = (packed ? q : v) + row * wkv + (packed ? (H + HK) * D : 0);
  // every element of q and k: rotary pairs (the first 2 * half dims) rotate, the rest pass through
  for (int i = threadIdx.x; i < (H + HK) * D; i += blockDim.x) {
    const bool isk = i >= H * D;
    const int hh = (isk ? i - H * D : i) / D, d = (isk ? i - H * D : i) % D;
    const T* src = (isk ? krow : qrow) + (size_t)hh * D;
    T* dst = (isk ? kr + row * HK * D : qr + row * H * D) + (size_t)hh * D;
    float y = to_f<T>(src[d]);
    if (rot && d < 2 * half) {
      int j, lo, hi;
      if (interleaved) j = d >> 1, lo = d & ~1, hi = lo + 1;
      else j = d < half ? d : d - half, lo = j, hi = j + half;
      const float c = to_f<T>(cos_c[(size_t)pos * half + j]), sn = to_f<T>(sin_c[(size_t)pos * half + j]);
      const float a = to_f<T>(src[lo]), bb = to_f<T>(src[hi]);
      y = d == lo ? a * c - bb * sn : bb * c + a * sn;
    }
    dst[d] = from_f<T>(y);
  }
  for (int i = threadIdx.x; i < HK * D; i += blockDim.x) vr[row * HK * D + i] = vrow[i];
}

// present rows [0, after) = work rows [write_start, write_start + after), rows [after, cap) zero
template <typename T>
__global__ void sliding_writeback_kernel(const T* __restrict__ wk, const T* __restrict__ wv, T* __restrict__ ok,
                                         T* __restrict__ ov, const SlidingGeo* __restrict__ geo, int HK, int cap,
                                         int wcap, int D) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.z, h = blockIdx.y;
  const SlidingGeo g = geo[b];
  const int cpr = D * (int)sizeof(T) / 16;
  const size_t src0 = ((size_t)b * HK + h) * wcap * D, dst0 = ((size_t)b * HK + h) * cap * D;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < cap * cpr; i += gridDim.x * blockDim.x) {
    const int r = i / cpr, c = i - r * cpr;
    const size_t dof = (dst0 + (size_t)r * D) * sizeof(T) + c * 16;
    uint4 vk = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
    if (r < g.after) {
      const size_t so = (src0 + (size_t)(g.write_start + r) * D) * sizeof(T) + c * 16;
      vk = *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(wk) + so);
      vv = *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(wv) + so);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<char*>(ok) + dof) = vk;
    *reinterpret_cast<uint4*>(reinterpret_cast<char*>(ov) + dof) = vv;
  }
}

struct SlidingLayout {
  size_t gqa, geo, seqw, qr, kr, vr, wk, wv, total;
};

b200ep_gqa_params inner_params(const b200ep_gqa_params& p) {
  b200ep_gqa_params ip = p;
  ip.cap = p.cap + p.seq;
  ip.do_rotary = 0;
  ip.packed_qkv = 0;
  return ip;
}

SlidingLayout sliding_layout(const b200ep_gqa_params& p, int esz) {
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  SlidingLayout l{};
  size_t o = 0;
  l.gqa = o, o += up(gqa_workspace_bytes(inner_params(p)));  // zeroed at allocation, left zeroed
  l.geo = o, o += up((size_t)p.batch * sizeof(SlidingGeo));
  l.seqw = o, o += up((size_t)p.batch * 4);
  l.qr = o, o += up((size_t)p.batch * p.seq * p.num_heads * p.head_size * esz);
  l.kr = o, o += up((size_t)p.batch * p.seq * p.kv_heads * p.head_size * esz);
  l.vr = o, o += up((size_t)p.batch * p.seq * p.kv_heads * p.head_size * esz);
  l.wk = o, o += up((size_t)p.batch * p.kv_heads * (p.cap + p.seq) * p.head_size * esz);
  l.wv = o, o += up((size_t)p.batch * p.kv_heads * (p.cap + p.seq) * p.head_size * esz);
  l.total = o;
  return l;
}

}  // namespace

size_t gqa_sliding_workspace_bytes(const b200ep_gqa_params& p, int dtype) {
  return sliding_layout(p, std::max(dtype_size(dtype), 2)).total;
}

int launch_gqa_sliding(const GqaSlidingArgs& a, cudaStream_t st) {
  const b200ep_gqa_params& p = a.p;
  B200EP_CHECK_ARG(p.batch > 0 && p.seq > 0 && p.num_heads > 0 && p.kv_heads > 0 && p.head_size > 0,
                   "GroupQueryAttention (sliding window cache): batch, seq, heads and head_size must be > 0");
  B200EP_CHECK_ARG(p.local_window > 0 && p.cap >= p.local_window,
                   "GroupQueryAttention: sliding cache requires 0 < local_window_size <= capacity");
  B200EP_CHECK_ARG(p.bias_batch == 0, "GroupQueryAttention: sliding_window_cache is incompatible with attention_bias");
  B200EP_CHECK_ARG(is_float_dtype(a.dtype), "GroupQueryAttention: dtype must be float32/float16/bfloat16");
  const int esz = dtype_size(a.dtype);
  B200EP_CHECK_ARG((p.head_size * esz) % 16 == 0, "GroupQueryAttention (sliding window cache): head_size * "
                                                  "element size must be a multiple of 16 bytes");
  B200EP_CHECK_ARG(a.query && a.past_key && a.past_value && a.present_key && a.present_value && a.seqlens_k &&
                       a.out && (p.packed_qkv || (a.key && a.value)),
                   "GroupQueryAttention (sliding window cache): null tensor pointer");
  if (p.do_rotary)
    B200EP_CHECK_ARG(a.cos_cache && a.sin_cache && p.rotary_half > 0 && 2 * p.rotary_half <= p.head_size &&
                         p.max_seq > 0,
                     "GroupQueryAttention: do_rotary needs cos/sin caches with 2*rotary_half <= head_size");
  const SlidingLayout l = sliding_layout(p, esz);
  B200EP_CHECK_ARG(a.workspace && a.workspace_bytes >= l.total,
                   "GroupQueryAttention (sliding window cache): workspace too small");
  B200EP_CHECK_ARG(p.batch <= 1024, "GroupQueryAttention (sliding window cache): batch > 1024");
  char* ws = static_cast<char*>(a.workspace);
  auto* geo = reinterpret_cast<SlidingGeo*>(ws + l.geo);
  auto* seqw = reinterpret_cast<int32_t*>(ws + l.seqw);
  const int B = (int)p.batch, S = (int)p.seq, H = (int)p.num_heads, HK = (int)p.kv_heads, D = (int)p.head_size;
  const int cap = (int)p.cap, wcap = cap + S;
  DeviceErrorSlot* err = device_error_slot();

  cudaError_t e = launch_k(sliding_geometry_kernel, dim3(1), dim3(std::min(1024, ((B + 31) / 32) * 32)), 0, st,
                           a.seqlens_k, B, S, cap, (int)p.local_window, geo, seqw);
  if (e != cudaSuccess) return cuda_status(e, "sliding-window geometry");
  const int cpr = D * esz / 16;
  const dim3 rgrid((unsigned)std::max(1, std::min(64, (cap * cpr + 255) / 256)), HK, B);
  e = by_float_dtype(a.dtype, [&](auto tag) {
    using T = decltype(tag);
    cudaError_t r = launch_k(sliding_seed_kernel<T>, rgrid, dim3(256), 0, st, static_cast<const T*>(a.past_key),
                             static_cast<const T*>(a.past_value), reinterpret_cast<T*>(ws + l.wk),
                             reinterpret_cast<T*>(ws + l.wv), geo, HK, cap, wcap, D);
    if (r != cudaSuccess) return r;
    return launch_k(sliding_rows_kernel<T>, dim3(S, B), dim3(256), 0, st, static_cast<const T*>(a.query),
                    static_cast<const T*>(a.key), static_cast<const T*>(a.value), (int)p.packed_qkv,
                    reinterpret_cast<T*>(ws + l.qr), reinterpret_cast<T*>(ws + l.kr), reinterpret_cast<T*>(ws + l.vr),
                    static_cast<const T*>(a.cos_cache), static_cast<const T*>(a.sin_cache), geo, S, H, HK, D,
                    (int)p.rotary_half, (int)p.interleaved, (int)p.do_rotary, (int)p.max_seq, err);
  });
  if (e != cudaSuccess) return cuda_status(e, "sliding-window staging");

  GqaArgs g{};
  g.p = inner_params(p);
  g.query = ws + l.qr;
  g.key = ws + l.kr;
  g.value = ws + l.vr;
  g.kv_key = ws + l.wk;
  g.kv_value = ws + l.wv;
  g.seqlens_k = seqw;
  g.out = a.out;
  g.dtype = a.dtype;
  g.workspace = ws + l.gqa;
  g.workspace_bytes = l.geo - l.gqa;
  if (int rc = launch_gqa(g, st)) return rc;

  e = by_float_dtype(a.dtype, [&](auto tag) {
    using T = decltype(tag);
    return launch_k(sliding_writeback_kernel<T>, rgrid, dim3(256), 0, st, reinterpret_cast<const T*>(ws + l.wk),
                    reinterpret_cast<const T*>(ws + l.wv), static_cast<T*>(a.present_key),
                    static_cast<T*>(a.present_value), geo, HK, cap, wcap, D);
  });
  if (e != cudaSuccess) return cuda_status(e, "sliding-window write-back");
  return B200EP_OK;
}

}  // namespace b200ep
