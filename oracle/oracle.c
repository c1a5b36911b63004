/*
 * CPU oracle for the int4 decode hot path — TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the arithmetic that the reference execution
 * provider (justinchuby/onnxruntime-mlx) maps onto ONNX Runtime's CPU EP
 * semantics for three operators:
 *
 *   - com.microsoft MatMulNBits         (rust/src/ops/quant.rs:986-1130)
 *   - com.microsoft GroupQueryAttention  (rust/src/ops/attention.rs:556-952)
 *   - SimplifiedLayerNormalization / RMSNormalization /
 *     SkipSimplifiedLayerNormalization    (rust/src/ops/norm.rs:163-246)
 *   - com.microsoft PagedAttention       (rust/src/ops/attention.rs:2495-2746)
 *
 * It is the checker for the CUDA kernels (tests, smoke(), and the timed CPU
 * baseline of bench.py).  The product library never links or calls it.
 *
 * Numeric conventions (chosen to model ORT CPU, the reference's parity target):
 *   - Dequantised weight = (float)(q - zp) * (float)scale, one fp32 multiply.
 *     This is the bit-exact target for every dequantising kernel.
 *   - Dot products / reductions accumulate in double; the result is rounded
 *     once to the I/O dtype.
 *   - fp16 / bf16 conversions use IEEE round-to-nearest-even.
 * The reference has no stored golden vectors for this path; the oracle is
 * pinned against fixtures generated from the reference's own test builders and
 * numpy references (tests/golden/gen_golden.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ONNX TensorProto element types (same values as ONNXTensorElementDataType). */
enum { OR_F32 = 1, OR_U8 = 2, OR_I32 = 6, OR_F16 = 10, OR_BF16 = 16 };

enum {
  OR_OK = 0,
  OR_EINVAL = 1,   /* bad argument / unsupported form */
  OR_ERANGE = 2    /* position or size outside the caches */
};

/* ---- fp16 / bf16 <-> fp32 (round to nearest even) ------------------------ */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float oracle_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  if (exp == 0) {
    if (man == 0) return u2f(sign);
    /* subnormal: value = man * 2^-24 */
    float v = (float)man * 5.9604644775390625e-08f;
    return sign ? -v : v;
  }
  if (exp == 31) return u2f(sign | 0x7f800000u | (man << 13));
  return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

uint16_t oracle_float_to_half(float f) {
  uint32_t u = f2u(f);
  uint32_t sign = (u >> 16) & 0x8000u;
  uint32_t a = u & 0x7fffffffu;
  if (a >= 0x7f800000u) /* inf or nan */
    return (uint16_t)(sign | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0u));
  if (a >= 0x477ff000u) /* rounds to >= 65520 -> inf */
    return (uint16_t)(sign | 0x7c00u);
  if (a < 0x38800000u) { /* result is subnormal or zero in fp16 */
    /* value / 2^-24, rounded to nearest even integer */
    float v = u2f(a) * 16777216.0f;
    float r = nearbyintf(v); /* default rounding mode is RNE */
    return (uint16_t)(sign | (uint32_t)r);
  }
  /* normal: rebias exponent, round mantissa from 23 to 10 bits */
  uint32_t mant_odd = (a >> 13) & 1u;
  a += 0xfffu + mant_odd;
  a -= (112u << 23);
  return (uint16_t)(sign | (a >> 13));
}

float oracle_bf16_to_float(uint16_t b) { return u2f((uint32_t)b << 16); }

uint16_t oracle_float_to_bf16(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

static inline float load_f(const void* p, int64_t i, int dt) {
  switch (dt) {
    case OR_F32: return ((const float*)p)[i];
    case OR_F16: return oracle_half_to_float(((const uint16_t*)p)[i]);
    case OR_BF16: return oracle_bf16_to_float(((const uint16_t*)p)[i]);
  }
  return NAN;
}

static inline void store_f(void* p, int64_t i, int dt, double v) {
  float f = (float)v;
  switch (dt) {
    case OR_F32: ((float*)p)[i] = f; break;
    case OR_F16: ((uint16_t*)p)[i] = oracle_float_to_half(f); break;
    case OR_BF16: ((uint16_t*)p)[i] = oracle_float_to_bf16(f); break;
  }
}

/* Round a float through the I/O dtype (identity for fp32). */
static inline float round_to(float v, int dt) {
  switch (dt) {
    case OR_F16: return oracle_half_to_float(oracle_float_to_half(v));
    case OR_BF16: return oracle_bf16_to_float(oracle_float_to_bf16(v));
  }
  return v;
}

static int is_float_dt(int dt) { return dt == OR_F32 || dt == OR_F16 || dt == OR_BF16; }

static void set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ---- MatMulNBits ----------------------------------------------------------
 * Layout (ORT contrib op; the reference's accepted forms, quant.rs:1655-1711):
 *   B       uint8 [N, nblocks, block*bits/8], values packed low-to-high along K
 *           (int4: low nibble = even k; quant.rs:675-698)
 *   scales  [N * nblocks], same float dtype as A
 *   zp      optional uint8; int4: [N, ceil(nblocks/2)] packed, low nibble =
 *           even block (quant.rs:906-919); int8: [N, nblocks].
 *           Absent -> 2^(bits-1) (quant.rs:821, 1107).
 *   K not a multiple of block: the tail of the last block is padding and the
 *   activation is zero-padded (quant.rs:1034-1039, 1074).
 */

static inline int mnb_q(const uint8_t* B, int64_t n, int64_t k, int64_t nblocks,
                        int bits, int block) {
  int64_t blob = (int64_t)block * bits / 8;
  int64_t blk = k / block, within = k % block;
  if (bits == 4) {
    uint8_t byte = B[(n * nblocks + blk) * blob + within / 2];
    return (within & 1) ? (byte >> 4) : (byte & 0x0f);
  }
  return B[(n * nblocks + blk) * blob + within];
}

static inline int mnb_zp(const uint8_t* zp, int64_t n, int64_t blk, int64_t nblocks,
                         int bits) {
  if (!zp) return 1 << (bits - 1);
  if (bits == 4) {
    int64_t cols = (nblocks + 1) / 2;
    uint8_t byte = zp[n * cols + blk / 2];
    return (blk & 1) ? (byte >> 4) : (byte & 0x0f);
  }
  return zp[n * nblocks + blk];
}

int oracle_matmulnbits_dequant(const uint8_t* B, const void* scales, int scale_dt,
                               const uint8_t* zp, int64_t N, int64_t K, int bits,
                               int block, float* W) {
  if (!B || !scales || !W || N <= 0 || K <= 0) return OR_EINVAL;
  if (bits != 4 && bits != 8) return OR_EINVAL;
  if (block < 16 || (block & (block - 1))) return OR_EINVAL;
  if (!is_float_dt(scale_dt)) return OR_EINVAL;
  int64_t nblocks = (K + block - 1) / block;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n)
    for (int64_t k = 0; k < K; ++k) {
      int64_t blk = k / block;
      float s = load_f(scales, n * nblocks + blk, scale_dt);
      int d = mnb_q(B, n, k, nblocks, bits, block) - mnb_zp(zp, n, blk, nblocks, bits);
      W[n * K + k] = (float)d * s;
    }
  return OR_OK;
}

int oracle_matmulnbits(const void* A, const uint8_t* B, const void* scales,
                       const uint8_t* zp, void* Y, int dt, int64_t M, int64_t N,
                       int64_t K, int bits, int block, int nthreads) {
  if (!A || !B || !scales || !Y || M < 0 || N <= 0 || K <= 0) return OR_EINVAL;
  if (!is_float_dt(dt)) return OR_EINVAL;
  if (bits != 4 && bits != 8) return OR_EINVAL;
  if (block < 16 || (block & (block - 1))) return OR_EINVAL;
  if (M == 0) return OR_OK;
  float* Af = (float*)malloc((size_t)M * (size_t)K * sizeof(float));
  if (!Af) return OR_EINVAL;
  set_threads(nthreads);
  for (int64_t i = 0; i < M * K; ++i) Af[i] = load_f(A, i, dt);
  const int64_t nblocks = (K + block - 1) / block;
  int failed = 0;
  /* one output row of W at a time: dequantise it (the same (float)(q - zp) * (float)scale as
     oracle_matmulnbits_dequant) into a per-thread buffer, then every token's dot product in double */
#pragma omp parallel reduction(| : failed)
  {
    float* w = (float*)malloc((size_t)K * sizeof(float));
    if (!w) failed = 1;
#pragma omp for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
      if (!w) continue;
      for (int64_t blk = 0; blk < nblocks; ++blk) {
        const float sc = load_f(scales, n * nblocks + blk, dt);
        const int z = mnb_zp(zp, n, blk, nblocks, bits);
        const int64_t k1 = (blk + 1) * block < K ? (blk + 1) * block : K;
        for (int64_t k = blk * block; k < k1; ++k)
          w[k] = (float)(mnb_q(B, n, k, nblocks, bits, block) - z) * sc;
      }
      for (int64_t m = 0; m < M; ++m) {
        const float* a = Af + m * K;
        double acc = 0.0;
        for (int64_t k = 0; k < K; ++k) acc += (double)a[k] * (double)w[k];
        store_f(Y, m * N + n, dt, acc);
      }
    }
    free(w);
  }
  free(Af);
  return failed ? OR_EINVAL : OR_OK;
}

/* ---- RMS norms ------------------------------------------------------------
 * y = x / sqrt(mean(x^2) + eps) * gamma over the last axis (norm.rs:163-183).
 * Skip form: r = x + skip; y = rms_norm(r) * gamma; residual output = r
 * (norm.rs:229-246).  The sum is kept in fp32 for the normalisation and
 * rounded to the I/O dtype only where it is written out.
 */

static void rms_row(const float* r, const void* gamma, void* Y, int64_t row,
                    int64_t hidden, float eps, int dt) {
  double ss = 0.0;
  for (int64_t j = 0; j < hidden; ++j) ss += (double)r[j] * (double)r[j];
  double inv = 1.0 / sqrt(ss / (double)hidden + (double)eps);
  for (int64_t j = 0; j < hidden; ++j)
    store_f(Y, row * hidden + j, dt, (double)r[j] * inv * (double)load_f(gamma, j, dt));
}

int oracle_rms_norm(const void* X, const void* gamma, void* Y, int dt, int64_t rows,
                    int64_t hidden, float eps, int nthreads) {
  if (!X || !gamma || !Y || rows < 0 || hidden <= 0 || !is_float_dt(dt)) return OR_EINVAL;
  set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < rows; ++i) {
    float* r = (float*)malloc((size_t)hidden * sizeof(float));
    for (int64_t j = 0; j < hidden; ++j) r[j] = load_f(X, i * hidden + j, dt);
    rms_row(r, gamma, Y, i, hidden, eps, dt);
    free(r);
  }
  return OR_OK;
}

int oracle_skip_rms_norm(const void* X, const void* skip, const void* gamma, void* Y,
                         void* residual_out, int dt, int64_t rows, int64_t hidden,
                         float eps, int nthreads) {
  if (!X || !skip || !gamma || !Y || rows < 0 || hidden <= 0 || !is_float_dt(dt))
    return OR_EINVAL;
  set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < rows; ++i) {
    float* r = (float*)malloc((size_t)hidden * sizeof(float));
    for (int64_t j = 0; j < hidden; ++j) {
      r[j] = load_f(X, i * hidden + j, dt) + load_f(skip, i * hidden + j, dt);
      if (residual_out) store_f(residual_out, i * hidden + j, dt, r[j]);
    }
    rms_row(r, gamma, Y, i, hidden, eps, dt);
    free(r);
  }
  return OR_OK;
}

/* ---- GroupQueryAttention --------------------------------------------------
 * Follows the reference handler (attention.rs:556-952) with ORT CPU's per-batch
 * sequence lengths:
 *   past_len_b = seqlens_k[b] + 1 - S          (the reference uses the uniform
 *                                               total_sequence_length - S,
 *                                               attention.rs:624-642; equal for
 *                                               uniform batches)
 *   query s sits at position past_len_b + s; it attends keys
 *   j <= past_len_b + s (lower-right causal, attention.rs:537-543) and, with a
 *   local window w > 0, keys j > past_len_b + s - w.
 *   RoPE from the cos/sin caches at those positions (attention.rs:417-461):
 *     non-interleaved: o1 = x1 c - x2 s, o2 = x2 c + x1 s on halves of the
 *     rotary dims; interleaved: the same on (even, odd) pairs; dims beyond
 *     2*half pass through.
 *   Optional per-head RMS norm of q/k (inputs 14/15) before RoPE
 *   (attention.rs:663-669).
 *   New K/V rows are written to present at [past_len_b, past_len_b + S)
 *   (shared buffer in place, attention.rs:893-902; growing concat 903-907).
 *   softmax(scale * q.k^T + bias) . V, scale = attr or 1/sqrt(D).
 * Rotated q / k are rounded to the I/O dtype before use, as ORT stores them.
 */

typedef struct {
  int64_t batch, seq, num_heads, kv_heads, head_size;
  int64_t past_cap;    /* axis-2 length of past_key/value (0 = no past) */
  int64_t present_cap; /* axis-2 length of present_key/value */
  int64_t max_seq;     /* rows of the cos/sin caches */
  int64_t rotary_half; /* cos_cache.shape[1] */
  int32_t do_rotary, interleaved, packed_qkv, shared_buffer;
  int32_t local_window;   /* <= 0: none */
  int32_t has_qk_norm;
  float scale;            /* 0 -> 1/sqrt(D) */
  float qk_norm_eps;
  int64_t bias_batch;     /* attention_bias batch dim (0 = absent, 1 = broadcast) */
  int64_t bias_total;     /* attention_bias last dim */
} oracle_gqa_params;

static void qk_norm_vec(float* x, int64_t d, const void* w, int dt, float eps) {
  double ss = 0.0;
  for (int64_t i = 0; i < d; ++i) ss += (double)x[i] * x[i];
  double inv = 1.0 / sqrt(ss / (double)d + (double)eps);
  for (int64_t i = 0; i < d; ++i) x[i] = (float)((double)x[i] * inv * load_f(w, i, dt));
}

static void rope_vec(float* x, int64_t d, int64_t half, int64_t pos, const void* cos_c,
                     const void* sin_c, int dt, int interleaved) {
  float tmp[1024];
  for (int64_t i = 0; i < d; ++i) tmp[i] = x[i];
  for (int64_t i = 0; i < half; ++i) {
    float c = load_f(cos_c, pos * half + i, dt);
    float s = load_f(sin_c, pos * half + i, dt);
    if (!interleaved) {
      float a = tmp[i], b = tmp[i + half];
      x[i] = a * c - b * s;
      x[i + half] = b * c + a * s;
    } else {
      float a = tmp[2 * i], b = tmp[2 * i + 1];
      x[2 * i] = a * c - b * s;
      x[2 * i + 1] = b * c + a * s;
    }
  }
}

int oracle_gqa(const oracle_gqa_params* p, const void* q, const void* k, const void* v,
               const void* past_k, const void* past_v, const int32_t* seqlens_k,
               const void* cos_c, const void* sin_c, const void* q_norm_w,
               const void* k_norm_w, const void* attn_bias, void* out, void* present_k,
               void* present_v, int dt, int nthreads) {
  if (!p || !q || !seqlens_k || !out || !present_k || !present_v || !is_float_dt(dt))
    return OR_EINVAL;
  const int64_t B = p->batch, S = p->seq, H = p->num_heads, HK = p->kv_heads,
                D = p->head_size;
  if (B <= 0 || S <= 0 || H <= 0 || HK <= 0 || D <= 0 || D > 1024 || H % HK) return OR_EINVAL;
  if (!p->packed_qkv && (!k || !v)) return OR_EINVAL;
  if (p->do_rotary && (!cos_c || !sin_c || 2 * p->rotary_half > D || p->rotary_half <= 0))
    return OR_EINVAL;
  if (p->has_qk_norm && (!q_norm_w || !k_norm_w)) return OR_EINVAL;
  const int64_t G = H / HK;
  const int64_t cap = p->present_cap;
  const int64_t qstride = p->packed_qkv ? (H + 2 * HK) * D : H * D;
  const int64_t kstride = p->packed_qkv ? qstride : HK * D;
  const float scale = p->scale != 0.0f ? p->scale : (float)(1.0 / sqrt((double)D));

  for (int64_t b = 0; b < B; ++b) {
    int64_t past_len = (int64_t)seqlens_k[b] + 1 - S;
    if (past_len < 0) return OR_ERANGE;
    if (past_len + S > cap) return OR_ERANGE;
    if (!p->shared_buffer && past_len > p->past_cap) return OR_ERANGE;
    if (p->do_rotary && past_len + S > p->max_seq) return OR_ERANGE;
  }

  /* 1. present = past (when not aliased), then append the new rows. */
  const int64_t esz = dt == OR_F32 ? 4 : 2;
  if (!p->shared_buffer) {
    memset(present_k, 0, (size_t)(B * HK * cap * D * esz));
    memset(present_v, 0, (size_t)(B * HK * cap * D * esz));
    if (p->past_cap > 0 && past_k && past_v) {
      int64_t rows = p->past_cap < cap ? p->past_cap : cap;
      for (int64_t b = 0; b < B; ++b)
        for (int64_t h = 0; h < HK; ++h) {
          size_t dst = (size_t)(((b * HK + h) * cap) * D * esz);
          size_t src = (size_t)(((b * HK + h) * p->past_cap) * D * esz);
          memcpy((char*)present_k + dst, (const char*)past_k + src, (size_t)(rows * D * esz));
          memcpy((char*)present_v + dst, (const char*)past_v + src, (size_t)(rows * D * esz));
        }
    }
  }

  /* 2. rotate + append new K and V; rotate Q into a scratch buffer. */
  float* qr = (float*)malloc((size_t)(B * S * H * D) * sizeof(float));
  if (!qr) return OR_EINVAL;
  for (int64_t b = 0; b < B; ++b) {
    int64_t past_len = (int64_t)seqlens_k[b] + 1 - S;
    for (int64_t s = 0; s < S; ++s) {
      int64_t pos = past_len + s;
      float vec[1024];
      for (int64_t h = 0; h < H; ++h) {
        for (int64_t i = 0; i < D; ++i) vec[i] = load_f(q, (b * S + s) * qstride + h * D + i, dt);
        if (p->has_qk_norm) qk_norm_vec(vec, D, q_norm_w, dt, p->qk_norm_eps);
        if (p->do_rotary)
          rope_vec(vec, D, p->rotary_half, pos, cos_c, sin_c, dt, p->interleaved);
        for (int64_t i = 0; i < D; ++i)
          qr[((b * S + s) * H + h) * D + i] = round_to(vec[i], dt);
      }
      for (int64_t h = 0; h < HK; ++h) {
        const void* ksrc = p->packed_qkv ? q : k;
        const void* vsrc = p->packed_qkv ? q : v;
        int64_t koff = p->packed_qkv ? H * D : 0;
        int64_t voff = p->packed_qkv ? (H + HK) * D : 0;
        for (int64_t i = 0; i < D; ++i)
          vec[i] = load_f(ksrc, (b * S + s) * kstride + koff + h * D + i, dt);
        if (p->has_qk_norm) qk_norm_vec(vec, D, k_norm_w, dt, p->qk_norm_eps);
        if (p->do_rotary)
          rope_vec(vec, D, p->rotary_half, pos, cos_c, sin_c, dt, p->interleaved);
        int64_t row = ((b * HK + h) * cap + pos) * D;
        for (int64_t i = 0; i < D; ++i) {
          store_f(present_k, row + i, dt, vec[i]);
          store_f(present_v, row + i, dt,
                  load_f(vsrc, (b * S + s) * kstride + voff + h * D + i, dt));
        }
      }
    }
  }

  /* 3. attention over the valid keys of present. */
  set_threads(nthreads);
#pragma omp parallel for schedule(dynamic) collapse(3)
  for (int64_t b = 0; b < B; ++b)
    for (int64_t h = 0; h < H; ++h)
      for (int64_t s = 0; s < S; ++s) {
        int64_t past_len = (int64_t)seqlens_k[b] + 1 - S;
        int64_t qpos = past_len + s;
        int64_t hk = h / G;
        int64_t lo = 0;
        if (p->local_window > 0 && qpos - p->local_window + 1 > 0)
          lo = qpos - p->local_window + 1;
        int64_t n = qpos + 1 - lo;
        double* sc = (double*)malloc((size_t)n * sizeof(double));
        const float* qv = qr + ((b * S + s) * H + h) * D;
        double mx = -INFINITY;
        for (int64_t j = lo; j <= qpos; ++j) {
          int64_t row = ((b * HK + hk) * cap + j) * D;
          double dot = 0.0;
          for (int64_t i = 0; i < D; ++i) dot += (double)qv[i] * load_f(present_k, row + i, dt);
          double x = dot * (double)scale;
          if (p->bias_batch > 0) {
            int64_t bb = p->bias_batch == 1 ? 0 : b;
            x += load_f(attn_bias, (bb * S + s) * p->bias_total + j, dt);
          }
          sc[j - lo] = x;
          if (x > mx) mx = x;
        }
        double den = 0.0;
        for (int64_t t = 0; t < n; ++t) {
          sc[t] = (mx == -INFINITY) ? 0.0 : exp(sc[t] - mx);
          den += sc[t];
        }
        for (int64_t i = 0; i < D; ++i) {
          double acc = 0.0;
          for (int64_t j = lo; j <= qpos; ++j)
            acc += sc[j - lo] * load_f(present_v, ((b * HK + hk) * cap + j) * D + i, dt);
          store_f(out, ((b * S + s) * H + h) * D + i, dt, den > 0 ? acc / den : 0.0);
        }
        free(sc);
      }
  free(qr);
  return OR_OK;
}

/* ---- GroupQueryAttention with a sliding-window KV cache -------------------
 * attention.rs:725-880 (sliding_window_cache = 1, local_window_size = W, capacity cap >= W;
 * claim 1552-1575), per batch b with S new rows:
 *   p      = max(seqlens_k[b] + 1 - S, 0)            absolute position of the first new row
 *   gap    = cap - W + 1
 *   end(L) = L if L <= cap, else L - gap * ceil((L - cap) / gap)   rows resident after L tokens
 *   before = end(p), after = end(p + S), kept = after - S, seed_offset = before - kept
 *   staging (any batch): kept < min(p, W - 1)
 *   work   = past[b, :, seed_start : before] ++ the new rows, seed_start = staging ? 0 : seed_offset
 *   query i (at work row seed_rows + i, seed_rows = before - seed_start) attends work rows
 *   [seed_rows + i - W + 1, seed_rows + i]; q and k are rotated at absolute positions p + i.
 *   present[b, :, 0 : after] = work[write_start : write_start + after], the rest zero,
 *   write_start = staging ? seed_offset : 0.
 * The attention over `work` is oracle_gqa's (shared buffer, no rotary, local window W). */
static int64_t sliding_end(int64_t len, int64_t cap, int64_t gap) {
  if (len <= cap) return len;
  return len - gap * ((len - cap + gap - 1) / gap);
}

int oracle_gqa_sliding(const oracle_gqa_params* p, const void* q, const void* k, const void* v,
                       const void* past_k, const void* past_v, const int32_t* seqlens_k,
                       const void* cos_c, const void* sin_c, void* out, void* present_k,
                       void* present_v, int dt, int nthreads) {
  if (!p || !q || !k || !v || !past_k || !past_v || !seqlens_k || !out || !present_k || !present_v ||
      !is_float_dt(dt) || p->packed_qkv || p->has_qk_norm || p->bias_batch)
    return OR_EINVAL;
  const int64_t B = p->batch, S = p->seq, H = p->num_heads, HK = p->kv_heads, D = p->head_size;
  const int64_t cap = p->past_cap, W = p->local_window;
  if (B <= 0 || S <= 0 || H <= 0 || HK <= 0 || D <= 0 || D > 1024 || H % HK) return OR_EINVAL;
  if (W <= 0 || cap < W || p->present_cap != cap) return OR_EINVAL;
  if (p->do_rotary && (!cos_c || !sin_c || 2 * p->rotary_half > D || p->rotary_half <= 0)) return OR_EINVAL;
  const int64_t gap = cap - W + 1, wcap = cap + S, esz = dt == OR_F32 ? 4 : 2;
  int64_t* geo = (int64_t*)malloc((size_t)B * 4 * sizeof(int64_t));
  int staging = 0;
  for (int64_t b = 0; b < B; ++b) {
    int64_t pp = (int64_t)seqlens_k[b] + 1 - S;
    if (pp < 0) pp = 0;
    const int64_t before = sliding_end(pp, cap, gap), after = sliding_end(pp + S, cap, gap);
    const int64_t kept = after - S, required = pp < W - 1 ? pp : W - 1;
    if (kept < required) staging = 1;
    if (p->do_rotary && pp + S > p->max_seq) { free(geo); return OR_ERANGE; }
    geo[4 * b + 0] = pp, geo[4 * b + 1] = before, geo[4 * b + 2] = after, geo[4 * b + 3] = before - kept;
  }
  char* wk = (char*)calloc((size_t)(B * HK * wcap * D), (size_t)esz);
  char* wv = (char*)calloc((size_t)(B * HK * wcap * D), (size_t)esz);
  char* qr = (char*)malloc((size_t)(B * S * H * D * esz));
  char* kr = (char*)malloc((size_t)(B * S * HK * D * esz));
  int32_t* seq_w = (int32_t*)malloc((size_t)B * sizeof(int32_t));
  /* work = the seed rows; q / k rotated at their absolute positions, rounded to the I/O dtype */
  for (int64_t b = 0; b < B; ++b) {
    const int64_t pp = geo[4 * b], before = geo[4 * b + 1], off = geo[4 * b + 3];
    const int64_t seed_start = staging ? 0 : off, seed_rows = before - seed_start;
    seq_w[b] = (int32_t)(seed_rows + S - 1);
    for (int64_t h = 0; h < HK; ++h) {
      const size_t src = (size_t)(((b * HK + h) * cap + seed_start) * D * esz);
      const size_t dst = (size_t)(((b * HK + h) * wcap) * D * esz);
      memcpy(wk + dst, (const char*)past_k + src, (size_t)(seed_rows * D * esz));
      memcpy(wv + dst, (const char*)past_v + src, (size_t)(seed_rows * D * esz));
    }
    for (int64_t s = 0; s < S; ++s) {
      float vec[1024];
      for (int64_t h = 0; h < H + HK; ++h) {
        const int isk = h >= H;
        const void* src = isk ? k : q;
        const int64_t hh = isk ? h - H : h, width = isk ? HK * D : H * D;
        for (int64_t i = 0; i < D; ++i) vec[i] = load_f(src, (b * S + s) * width + hh * D + i, dt);
        if (p->do_rotary) rope_vec(vec, D, p->rotary_half, pp + s, cos_c, sin_c, dt, p->interleaved);
        for (int64_t i = 0; i < D; ++i)
          store_f(isk ? (void*)kr : (void*)qr, (b * S + s) * width + hh * D + i, dt, vec[i]);
      }
    }
  }
  oracle_gqa_params ap = *p;
  ap.past_cap = ap.present_cap = wcap;
  ap.do_rotary = 0;
  ap.shared_buffer = 1;
  ap.local_window = (int32_t)W;
  int rc = oracle_gqa(&ap, qr, kr, v, wk, wv, seq_w, NULL, NULL, NULL, NULL, NULL, out, wk, wv, dt, nthreads);
  if (rc == OR_OK) {
    memset(present_k, 0, (size_t)(B * HK * cap * D * esz));
    memset(present_v, 0, (size_t)(B * HK * cap * D * esz));
    for (int64_t b = 0; b < B; ++b) {
      const int64_t after = geo[4 * b + 2], ws = staging ? geo[4 * b + 3] : 0;
      for (int64_t h = 0; h < HK; ++h) {
        const size_t src = (size_t)(((b * HK + h) * wcap + ws) * D * esz);
        const size_t dst = (size_t)(((b * HK + h) * cap) * D * esz);
        memcpy((char*)present_k + dst, wk + src, (size_t)(after * D * esz));
        memcpy((char*)present_v + dst, wv + src, (size_t)(after * D * esz));
      }
    }
  }
  free(geo), free(wk), free(wv), free(qr), free(kr), free(seq_w);
  return rc;
}

/* ---- PagedAttention (com.microsoft) ---------------------------------------
 * paged_attention_op, attention.rs:2495-2746 (SEPARATE K / V caches, no
 * slot_mapping / head_sink / q-k norm, rotary_offset 0):
 *   sequence b owns packed rows [cum[b], cum[b+1]) and follows past[b] cached
 *   tokens; row j sits at position p = past[b] + j (2588-2596);
 *   RoPE of the new q and k at those positions, in the I/O dtype (2619-2624);
 *   the new k / v rows are scattered into physical block bt[b][p / bs], row
 *   p % bs of the caches [num_blocks, bs, kv_heads, D] (2632-2675);
 *   keys 0 .. past[b]-1 are gathered from the cache through the block table and
 *   the new rows appended (2678-2700); query j attends keys <= past[b] + j with
 *   an fp32 softmax (causal_mask_topleft with offset past, 2703-2711);
 *   scale = attr or 1/sqrt(D) (attr_scale).  Output [num_tokens, H * D].
 * Rotated q / k are rounded to the I/O dtype before use. */
typedef struct {
  int64_t batch, num_tokens, num_heads, kv_heads, head_size;
  int64_t num_blocks, block_size, max_blocks;
  int64_t max_seq, rotary_half;
  int32_t do_rotary, interleaved;
  float scale;
} oracle_paged_params;

static int64_t paged_slot(const oracle_paged_params* p, const int32_t* bt, int64_t b, int64_t pos) {
  int64_t blk = pos / p->block_size;
  if (pos < 0 || blk >= p->max_blocks) return -1;
  int64_t phys = bt[b * p->max_blocks + blk];
  if (phys < 0 || phys >= p->num_blocks) return -1;
  return phys * p->block_size + pos % p->block_size;
}

int oracle_paged_attention(const oracle_paged_params* p, const void* q, const void* k,
                           const void* v, void* kc, void* vc, const int32_t* cum,
                           const int32_t* past, const int32_t* bt, const void* cos_c,
                           const void* sin_c, void* out, int dt, int nthreads) {
  if (!p || !q || !k || !v || !kc || !vc || !cum || !past || !bt || !out || !is_float_dt(dt))
    return OR_EINVAL;
  const int64_t B = p->batch, T = p->num_tokens, H = p->num_heads, HK = p->kv_heads,
                D = p->head_size;
  if (B <= 0 || T < 0 || H <= 0 || HK <= 0 || D <= 0 || D > 1024 || H % HK) return OR_EINVAL;
  if (p->block_size <= 0 || p->num_blocks <= 0 || p->max_blocks <= 0) return OR_EINVAL;
  if (p->do_rotary && (!cos_c || !sin_c || p->rotary_half <= 0 || 2 * p->rotary_half > D))
    return OR_EINVAL;
  if (cum[0] != 0 || cum[B] != T) return OR_EINVAL;
  for (int64_t b = 0; b < B; ++b) {
    if (cum[b + 1] < cum[b] || past[b] < 0) return OR_EINVAL;
    int64_t total = (int64_t)past[b] + (cum[b + 1] - cum[b]);
    for (int64_t pos = 0; pos < total; ++pos)
      if (paged_slot(p, bt, b, pos) < 0) return OR_ERANGE;
    if (p->do_rotary && cum[b + 1] > cum[b] && total > p->max_seq) return OR_ERANGE;
  }
  const int64_t G = H / HK, row = HK * D;
  const float scale = p->scale != 0.0f ? p->scale : (float)(1.0 / sqrt((double)D));

  /* 1. rotate q into scratch; rotate k and scatter k / v into the caches. */
  float* qr = (float*)malloc((size_t)((T > 0 ? T : 1) * H * D) * sizeof(float));
  if (!qr) return OR_EINVAL;
  for (int64_t b = 0; b < B; ++b)
    for (int64_t t = cum[b]; t < cum[b + 1]; ++t) {
      int64_t pos = (int64_t)past[b] + (t - cum[b]);
      float vec[1024];
      for (int64_t h = 0; h < H; ++h) {
        for (int64_t i = 0; i < D; ++i) vec[i] = load_f(q, t * H * D + h * D + i, dt);
        if (p->do_rotary) rope_vec(vec, D, p->rotary_half, pos, cos_c, sin_c, dt, p->interleaved);
        for (int64_t i = 0; i < D; ++i) qr[(t * H + h) * D + i] = round_to(vec[i], dt);
      }
      int64_t slot = paged_slot(p, bt, b, pos);
      for (int64_t h = 0; h < HK; ++h) {
        for (int64_t i = 0; i < D; ++i) vec[i] = load_f(k, t * row + h * D + i, dt);
        if (p->do_rotary) rope_vec(vec, D, p->rotary_half, pos, cos_c, sin_c, dt, p->interleaved);
        for (int64_t i = 0; i < D; ++i) {
          store_f(kc, slot * row + h * D + i, dt, vec[i]);
          store_f(vc, slot * row + h * D + i, dt, load_f(v, t * row + h * D + i, dt));
        }
      }
    }

  /* 2. causal attention of every packed row over its sequence's keys. */
  set_threads(nthreads);
#pragma omp parallel for schedule(dynamic) collapse(2)
  for (int64_t t = 0; t < T; ++t)
    for (int64_t h = 0; h < H; ++h) {
      int64_t b = 0;
      while (b + 1 < B && cum[b + 1] <= t) ++b;
      int64_t qpos = (int64_t)past[b] + (t - cum[b]);
      int64_t hk = h / G, n = qpos + 1;
      double* sc = (double*)malloc((size_t)n * sizeof(double));
      const float* qv = qr + (t * H + h) * D;
      double mx = -INFINITY;
      for (int64_t j = 0; j < n; ++j) {
        int64_t slot = paged_slot(p, bt, b, j);
        double dot = 0.0;
        for (int64_t i = 0; i < D; ++i) dot += (double)qv[i] * load_f(kc, slot * row + hk * D + i, dt);
        sc[j] = dot * (double)scale;
        if (sc[j] > mx) mx = sc[j];
      }
      double den = 0.0;
      for (int64_t j = 0; j < n; ++j) {
        sc[j] = exp(sc[j] - mx);
        den += sc[j];
      }
      for (int64_t i = 0; i < D; ++i) {
        double acc = 0.0;
        for (int64_t j = 0; j < n; ++j)
          acc += sc[j] * load_f(vc, paged_slot(p, bt, b, j) * row + hk * D + i, dt);
        store_f(out, (t * H + h) * D + i, dt, acc / den);
      }
      free(sc);
    }
  free(qr);
  return OR_OK;
}

/* ---- GatherBlockQuantized (int4, gather_axis 0, quantize_axis last) -------
 * Row gather then (q - zp) * scale, zp default 8 (quant.rs:1134-1200). */
int oracle_gather_block_quantized(const uint8_t* data, const void* scales, int scale_dt,
                                  const uint8_t* zp, const int64_t* indices,
                                  int64_t n_indices, int64_t vocab, int64_t dim,
                                  int block, void* out, int out_dt) {
  if (!data || !scales || !indices || !out || dim % block || dim % 2) return OR_EINVAL;
  int64_t nblocks = dim / block;
  for (int64_t i = 0; i < n_indices; ++i) {
    int64_t r = indices[i];
    if (r < 0) r += vocab;
    if (r < 0 || r >= vocab) return OR_ERANGE;
    for (int64_t j = 0; j < dim; ++j) {
      uint8_t byte = data[r * (dim / 2) + j / 2];
      int qv = (j & 1) ? (byte >> 4) : (byte & 0x0f);
      int64_t blk = j / block;
      int z = 8;
      if (zp) {
        uint8_t zb = zp[r * ((nblocks + 1) / 2) + blk / 2];
        z = (blk & 1) ? (zb >> 4) : (zb & 0x0f);
      }
      float s = load_f(scales, r * nblocks + blk, scale_dt);
      store_f(out, i * dim + j, out_dt, (double)((float)(qv - z) * s));
    }
  }
  return OR_OK;
}
