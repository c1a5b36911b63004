// Claim predicates for the hot path (MatMulNBits, GroupQueryAttention, the RMS norms) and the
// elementwise glue a Llama-style decoder layer needs so that its partition does not fragment.
// Each predicate restates the accept/reject rules of the reference claim it names.
#include "registry.h"

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>

namespace b200ep {

namespace {

constexpr int kF32 = 1, kU8 = 2, kI32 = 6, kI64 = 7, kF16 = 10, kBF16 = 16;

const char* dtype_name(int dt) {
  switch (dt) {
    case kF32: return "float32";
    case kU8: return "uint8";
    case kI32: return "int32";
    case kI64: return "int64";
    case kF16: return "float16";
    case kBF16: return "bfloat16";
    case 0: return "unknown";
  }
  return "other";
}

std::string fmt(const char* f, ...) __attribute__((format(printf, 1, 2)));
std::string fmt(const char* f, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, f);
  vsnprintf(buf, sizeof buf, f, ap);
  va_end(ap);
  return buf;
}

#define REQUIRE(cond, ...) \
  do {                     \
    if (!(cond)) return ClaimResult::no(fmt(__VA_ARGS__)); \
  } while (0)

int in_dt(const NodeView& v, size_t i) {
  auto* info = v.input_info(i);
  return info ? info->dtype : 0;
}
int out_dt(const NodeView& v, size_t i) {
  auto* info = v.output_info(i);
  return info ? info->dtype : 0;
}

// ---- MatMulNBits: rust/src/ops/quant.rs:1655-1711 ------------------------------------------
ClaimResult matmulnbits_claim(const NodeView& v) {
  REQUIRE(v.num_outputs() >= 1, "requires at least one output");
  const int o = out_dt(v, 0);
  REQUIRE(is_ep_float(o), "output must be a float (fp32/fp16/bf16), got %s", dtype_name(o));
  REQUIRE(v.input_info(0) && v.input_info(1) && v.input_info(2), "missing tensor type/shape info on an input");
  const int a = in_dt(v, 0), b = in_dt(v, 1), s = in_dt(v, 2);
  REQUIRE(is_ep_float(a) && b == kU8 && is_ep_float(s),
          "activation/scales must be float and packed weights uint8, got a=%s, b=%s, scales=%s",
          dtype_name(a), dtype_name(b), dtype_name(s));
  REQUIRE(a == s && a == o, "activation, scales and output must share one float dtype, got a=%s, scales=%s, out=%s",
          dtype_name(a), dtype_name(s), dtype_name(o));
  if (v.input_present(3)) REQUIRE(in_dt(v, 3) == kU8, "zero_points must be uint8 when present");
  for (size_t i = 4; i < v.num_inputs(); ++i)
    REQUIRE(!v.input_present(i), "g_idx and bias inputs are not supported");
  const int64_t bits = v.int_attr("bits", 4), block = v.int_attr("block_size", 32);
  REQUIRE(bits == 4 || bits == 8, "only 4-bit and 8-bit weights are supported");
  REQUIRE(block == 16 || block == 32 || block == 64 || block == 128,
          "block_size must be 16, 32, 64, or 128 (got %lld)", (long long)block);
  // The device path keeps the weights resident: they must be initializers (the reference caches
  // constant weights the same way, quant.rs:634-710).
  REQUIRE(v.const_input(1) && v.const_input(2) && (!v.input_present(3) || v.const_input(3)),
          "B, scales and zero_points must be initializers");
  REQUIRE(v.int_attr("K", 0) > 0 && v.int_attr("N", 0) > 0, "attributes K and N are required");
  return ClaimResult::yes();
}

// ---- GroupQueryAttention: rust/src/ops/attention.rs:1520-1738 --------------------------------
ClaimResult gqa_claim(const NodeView& v) {
  REQUIRE(v.num_outputs() > 0, "requires at least 1 output");
  const int o = out_dt(v, 0);
  REQUIRE(is_ep_float(o), "output must have a float dtype, got %s", dtype_name(o));
  const size_t nin = v.num_inputs();
  REQUIRE(nin >= 7 && nin <= 16, "expects 7 required inputs plus optional rotary/bias/QK-norm inputs, got %zu", nin);
  const bool sliding = v.int_attr("sliding_window_cache", 0) != 0;
  const bool has_bias = v.input_present(10);
  if (sliding) {  // attention.rs:1552-1575
    const int64_t window = v.int_attr("local_window_size", -1);
    REQUIRE(window > 0, "sliding_window_cache=1 requires local_window_size > 0");
    REQUIRE(!has_bias, "sliding_window_cache is incompatible with attention_bias");
    REQUIRE(v.output_present(1) && v.output_present(2), "sliding_window_cache requires present key/value outputs");
    auto* pk = v.input_info(3);
    auto* pv = v.input_info(4);
    REQUIRE(pk && pk->shape.size() == 4 && pk->shape[2] >= window,
            "sliding-window key cache capacity must be at least local_window_size");
    REQUIRE(pv && pv->shape.size() == 4 && pv->shape[2] >= window,
            "sliding-window value cache capacity must be at least local_window_size");
    REQUIRE(!v.input_present(14), "sliding_window_cache with q/k norm weights is not implemented on this EP");
  }
  const bool do_rotary = v.int_attr("do_rotary", 1) != 0;
  REQUIRE(nin != 7 || !do_rotary, "7-input GroupQueryAttention requires do_rotary=0 because cos/sin caches are absent");
  const bool packed = v.input_present(0) && !v.input_present(1) && !v.input_present(2);
  REQUIRE(packed || (v.input_present(0) && v.input_present(1) && v.input_present(2)),
          "Q/K/V must be either all separate or packed in input 0 with inputs 1 and 2 absent");
  REQUIRE(v.input_present(3) && v.input_present(4), "past_key/past_value are required on this EP");
  std::vector<size_t> fidx = packed ? std::vector<size_t>{0, 3, 4} : std::vector<size_t>{0, 1, 2, 3, 4};
  if (do_rotary) {
    REQUIRE(v.input_present(7) && v.input_present(8), "do_rotary=1 requires cos_cache and sin_cache");
    fidx.push_back(7);
    fidx.push_back(8);
  }
  if (has_bias) fidx.push_back(10);
  if (v.input_present(14)) {
    fidx.push_back(14);
    fidx.push_back(15);
  }
  for (size_t i : fidx) {
    REQUIRE(v.input_info(i), "input %zu lacks tensor type/shape info", i);
    REQUIRE(in_dt(v, i) == o, "input %zu must have output dtype %s, got %s", i, dtype_name(o), dtype_name(in_dt(v, i)));
  }
  for (size_t i = 1; i < v.num_outputs() && i < 3; ++i) {
    if (!v.output_present(i)) continue;
    REQUIRE(out_dt(v, i) == o, "output %zu must have dtype %s, got %s", i, dtype_name(o), dtype_name(out_dt(v, i)));
  }
  for (size_t i : {5, 6}) {
    REQUIRE(v.input_info(i), "input %zu lacks tensor type/shape info", i);
    REQUIRE(in_dt(v, i) == kI32, "input %zu must have int32 dtype, got %s", i, dtype_name(in_dt(v, i)));
  }
  if (has_bias) {
    auto* bias = v.input_info(10);
    REQUIRE(bias && bias->shape.size() == 4, "attention_bias (input 10) must have rank 4");
  }
  const int64_t nh = v.int_attr("num_heads", 0), kvh = v.int_attr("kv_num_heads", 0);
  REQUIRE(nh > 0 && kvh > 0 && nh % kvh == 0, "num_heads (%lld) must be a positive multiple of kv_num_heads (%lld)",
          (long long)nh, (long long)kvh);
  auto* q = v.input_info(0);
  REQUIRE(q && q->shape.size() == 3 && q->shape[2] > 0, "query must have rank 3 with a static hidden size");
  int64_t head;
  if (packed) {
    REQUIRE(q->shape[2] % (nh + 2 * kvh) == 0, "packed QKV hidden size (%lld) must be divisible by total heads (%lld)",
            (long long)q->shape[2], (long long)(nh + 2 * kvh));
    head = q->shape[2] / (nh + 2 * kvh);
  } else {
    REQUIRE(q->shape[2] % nh == 0, "query hidden size must be divisible by num_heads");
    head = q->shape[2] / nh;
  }
  REQUIRE(head <= 256, "head_size %lld > 256 is not supported", (long long)head);
  auto* pk = v.input_info(3);
  REQUIRE(pk && pk->shape.size() == 4, "past_key must have rank 4 [B, kv_heads, cap, head]");
  REQUIRE(!v.input_present(9) || !do_rotary, "custom position_ids with in-op rotary are unsupported");
  REQUIRE(!v.input_present(11), "head_sink/smooth softmax is unsupported");
  REQUIRE(!v.input_present(12) && !v.input_present(13), "quantized KV cache scales are unsupported");
  REQUIRE(v.string_attr("k_quant_type", "NONE") == "NONE" && v.string_attr("v_quant_type", "NONE") == "NONE",
          "quantized KV cache is unsupported");
  REQUIRE(v.input_present(14) == v.input_present(15), "q_norm_weight and k_norm_weight must be provided together");
  if (v.input_present(14)) {
    for (size_t i : {14, 15}) {
      auto* w = v.input_info(i);
      REQUIRE(w && w->shape.size() == 1 && w->shape[0] == head, "Q/K norm weight %zu must have shape [head_size=%lld]",
              i, (long long)head);
    }
  }
  if (do_rotary) {
    auto* cc = v.input_info(7);
    REQUIRE(cc && cc->shape.size() == 2 && cc->shape[1] > 0 && 2 * cc->shape[1] <= head && cc->shape[1] <= 128,
            "cos_cache must be [max_seq, rotary_dim/2] with rotary_dim <= head_size");
  }
  REQUIRE(v.int_attr("smooth_softmax", 0) != 1, "smooth_softmax=1 is unsupported");
  REQUIRE(v.int_attr("qk_output", 0) == 0, "qk_output is unsupported");
  REQUIRE(v.float_attr("softcap", 0.f) == 0.f, "softcap is unsupported");
  return ClaimResult::yes();
}

// ---- norms: rust/src/ops/norm.rs:460-610 ---------------------------------------------------
ClaimResult rms_norm_claim(const NodeView& v) {
  REQUIRE(v.num_inputs() == 2 && v.num_outputs() > 0, "expects 2 inputs and at least 1 output, got %zuin/%zuout",
          v.num_inputs(), v.num_outputs());
  auto* x = v.input_info(0);
  REQUIRE(x && v.input_info(1) && v.output_info(0), "missing tensor type/shape info on an input or the first output");
  REQUIRE(is_ep_float(x->dtype) && in_dt(v, 1) == x->dtype && out_dt(v, 0) == x->dtype,
          "X, scale, and output must share one float dtype, got %s, %s -> %s", dtype_name(x->dtype),
          dtype_name(in_dt(v, 1)), dtype_name(out_dt(v, 0)));
  REQUIRE(v.int_attr("axis", -1) == -1, "only axis=-1 is supported");
  REQUIRE(x->shape.empty() || x->shape.back() <= 8192, "hidden size > 8192 is not supported");
  return ClaimResult::yes();
}

ClaimResult simplified_layer_norm_claim(const NodeView& v) {
  REQUIRE(v.num_inputs() == 2 && v.num_outputs() == 1, "expects 2 inputs and 1 output, got %zuin/%zuout",
          v.num_inputs(), v.num_outputs());
  auto* x = v.input_info(0);
  REQUIRE(x && v.input_info(1) && v.output_info(0), "missing tensor type/shape info on an input or the output");
  REQUIRE(is_ep_float(x->dtype) && in_dt(v, 1) == x->dtype && out_dt(v, 0) == x->dtype,
          "X, scale, and output must share one float dtype");
  REQUIRE(!x->shape.empty(), "input must have rank >= 1 (got a scalar)");
  const int64_t axis = v.int_attr("axis", -1);
  REQUIRE(axis == -1 || axis == (int64_t)x->shape.size() - 1, "only the last axis is supported (got axis=%lld)",
          (long long)axis);
  REQUIRE(x->shape.back() <= 8192, "hidden size > 8192 is not supported");
  return ClaimResult::yes();
}

ClaimResult skip_rms_norm_claim(const NodeView& v) {
  REQUIRE(v.num_inputs() == 3 && v.num_outputs() > 0, "expects 3 inputs and at least 1 output, got %zuin/%zuout",
          v.num_inputs(), v.num_outputs());
  auto* x = v.input_info(0);
  REQUIRE(x && v.output_info(0), "missing tensor type/shape info on X or the first output");
  REQUIRE(is_ep_float(x->dtype) && out_dt(v, 0) == x->dtype, "X and output must share one float dtype");
  REQUIRE(in_dt(v, 1) == x->dtype, "skip must match X dtype");
  REQUIRE(in_dt(v, 2) == x->dtype, "gamma must match X dtype");
  REQUIRE(!x->shape.empty() && x->shape.back() <= 8192, "hidden size > 8192 is not supported");
  // mean (out[1]) / inv-std (out[2]) are accepted but never produced: a consumer of them makes
  // them partition outputs and compilation fails loudly (norm.rs:582-589).
  return ClaimResult::yes();
}

// ---- GatherBlockQuantized (int4 embedding), rust/src/ops/quant.rs:1713-1749 -----------------
ClaimResult gbq_claim(const NodeView& v) {
  REQUIRE(v.num_outputs() >= 1 && v.num_inputs() >= 3, "expects data, indices, scales");
  REQUIRE(in_dt(v, 0) == kU8, "data must be uint8 packed int4");
  REQUIRE(in_dt(v, 1) == kI32 || in_dt(v, 1) == kI64, "indices must be int32/int64");
  REQUIRE(is_ep_float(in_dt(v, 2)) && out_dt(v, 0) == in_dt(v, 2), "scales and output must share one float dtype");
  REQUIRE(v.int_attr("bits", 4) == 4, "only 4-bit data is supported");
  REQUIRE(v.int_attr("gather_axis", 0) == 0, "only gather_axis=0 is supported");
  auto* d = v.input_info(0);
  REQUIRE(d && d->shape.size() == 2, "data must be rank 2 [rows, dim/2]");
  REQUIRE(v.int_attr("quantize_axis", 1) == 1, "only quantize_axis=1 is supported");
  const int64_t block = v.int_attr("block_size", 128);
  REQUIRE(block >= 16 && (block & (block - 1)) == 0 && (2 * d->shape[1]) % block == 0,
          "block_size must be a power of two >= 16 dividing the row");
  REQUIRE(v.const_input(0) && v.const_input(2) && (!v.input_present(3) || v.const_input(3)),
          "data, scales and zero_points must be initializers");
  return ClaimResult::yes();
}

// ---- elementwise glue: rust/src/ops/elementwise.rs:925-985 ---------------------------------
bool broadcastable(const ValueInfo* a, const ValueInfo* b) {
  if (!a || !b) return false;
  const size_t n = std::max(a->shape.size(), b->shape.size());
  if (n > 6) return false;
  for (size_t i = 0; i < n; ++i) {
    int64_t da = i < a->shape.size() ? a->shape[a->shape.size() - 1 - i] : 1;
    int64_t db = i < b->shape.size() ? b->shape[b->shape.size() - 1 - i] : 1;
    if (da != db && da != 1 && db != 1 && da != -1 && db != -1) return false;
  }
  return true;
}

ClaimResult binary_claim(const NodeView& v) {
  REQUIRE(v.num_inputs() == 2 && v.num_outputs() == 1, "expects 2 inputs and 1 output");
  const int o = out_dt(v, 0);
  REQUIRE(is_ep_float(o) || is_ep_int(o), "float or int32 / int64 output required, got %s", dtype_name(o));
  REQUIRE(in_dt(v, 0) == o && in_dt(v, 1) == o, "inputs must share the output dtype");
  REQUIRE(broadcastable(v.input_info(0), v.input_info(1)), "inputs must be broadcastable with rank <= 6");
  return ClaimResult::yes();
}

ClaimResult sigmoid_claim(const NodeView& v) {
  REQUIRE(v.num_inputs() == 1 && v.num_outputs() == 1, "expects 1 input and 1 output");
  REQUIRE(is_ep_float(out_dt(v, 0)) && in_dt(v, 0) == out_dt(v, 0), "float input/output of one dtype required");
  return ClaimResult::yes();
}

ClaimResult cast_claim(const NodeView& v) {
  REQUIRE(v.num_inputs() == 1 && v.num_outputs() == 1, "expects 1 input and 1 output");
  const int i = in_dt(v, 0), o = out_dt(v, 0);
  REQUIRE((is_ep_float(i) && is_ep_float(o)) || (is_ep_int(i) && is_ep_int(o)),
          "only float <-> float and int32 / int64 <-> int32 / int64 casts are claimed");
  REQUIRE(v.int_attr("to", 0) == o, "'to' must match the output dtype");
  return ClaimResult::yes();
}

// ---- integer glue of exported decoders ------------------------------------------------------
// The attention-mask chain of a GenAI-exported decoder: seqlens_k = Cast(Sub(ReduceSum(mask, 1), 1))
// and total_sequence_length = Cast(Gather(Shape(mask), 1)) (rust/src/compiled.rs:385-430 reads the
// same two quantities).  Claimed for int32 / int64 tensors only, where they are glue rather than
// model math; everything whose value is known on the host is evaluated there by the plan.

int norm_axis(int64_t a, int64_t rank) { return (int)(a < 0 ? a + rank : a); }

// Shape: rust/src/ops/shape.rs:2071-2109 (1-D int64 output of the sliced rank interval)
ClaimResult shape_claim(const NodeView& v) {
  REQUIRE(v.num_inputs() == 1 && v.num_outputs() == 1, "Shape expects 1 input and 1 output, got %zuin/%zuout",
          v.num_inputs(), v.num_outputs());
  auto* d = v.input_info(0);
  REQUIRE(d, "missing data tensor type/shape info");
  auto* o = v.output_info(0);
  REQUIRE(o && o->dtype == kI64 && o->shape.size() == 1, "Shape: output must be a 1-D int64 tensor");
  const int64_t rank = (int64_t)d->shape.size();
  int64_t s = v.int_attr("start", 0), e = v.int_attr("end", rank);
  s = std::clamp<int64_t>(s < 0 ? s + rank : s, 0, rank);
  e = std::clamp<int64_t>(e < 0 ? e + rank : e, 0, rank);
  REQUIRE(o->shape[0] < 0 || o->shape[0] == std::max<int64_t>(e - s, 0),
          "Shape: output extent %lld must equal the sliced rank interval %lld (start..end)", (long long)o->shape[0],
          (long long)std::max<int64_t>(e - s, 0));
  return ClaimResult::yes();
}

// Gather over a 1-D integer vector with constant indices (shape.rs:1169-1201 for the general form)
ClaimResult gather_claim(const NodeView& v) {
  REQUIRE(v.num_inputs() == 2 && v.num_outputs() == 1, "Gather expects 2 inputs and 1 output");
  auto* d = v.input_info(0);
  REQUIRE(d && is_ep_int(d->dtype) && d->shape.size() == 1,
          "only 1-D int32 / int64 data (shape vectors) is gathered on the EP");
  REQUIRE(norm_axis(v.int_attr("axis", 0), 1) == 0, "axis must be 0 for 1-D data");
  const Initializer* idx = v.const_input(1);
  REQUIRE(idx && (idx->dtype == kI32 || idx->dtype == kI64) && idx->shape.size() <= 1 && idx->numel() <= 8,
          "indices must be a constant int32 / int64 scalar or vector of at most 8 entries");
  REQUIRE(out_dt(v, 0) == d->dtype, "output dtype must equal the data dtype");
  return ClaimResult::yes();
}

// ReduceSum over the last axis of an integer tensor (reduction.rs:894; the mask's key axis)
ClaimResult reduce_sum_claim(const NodeView& v) {
  REQUIRE(v.num_outputs() == 1, "ReduceSum expects 1 output");
  auto* d = v.input_info(0);
  REQUIRE(d && is_ep_int(d->dtype) && !d->shape.empty(), "only int32 / int64 data of rank >= 1 is reduced on the EP");
  REQUIRE(out_dt(v, 0) == d->dtype, "output dtype must equal the data dtype");
  std::vector<int64_t> axes;
  if (v.since_version() >= 13) {
    REQUIRE(v.input_present(1), "axes input required (reducing every axis is not claimed)");
    const Initializer* a = v.const_input(1);
    REQUIRE(a, "axes must be a constant initializer");
    axes = const_ints(a);
  } else {
    axes = v.ints_attr("axes");
  }
  const int64_t rank = (int64_t)d->shape.size();
  REQUIRE(axes.size() == 1 && norm_axis(axes[0], rank) == rank - 1, "only a reduction over the last axis is claimed");
  return ClaimResult::yes();
}

// Unsqueeze / Squeeze / Reshape of integer tensors with constant axes / shape (shape.rs:1646-1745):
// the values pass through unchanged
ClaimResult int_layout_claim(const NodeView& v) {
  REQUIRE(v.num_outputs() == 1, "%s expects 1 output", v.op_type().c_str());
  auto* d = v.input_info(0);
  REQUIRE(d && is_ep_int(d->dtype), "only int32 / int64 tensors are reshaped on the EP");
  REQUIRE(out_dt(v, 0) == d->dtype, "output dtype must equal the data dtype");
  const bool axes_input = v.op_type() == "Reshape" || v.since_version() >= 13;
  if (axes_input) {
    REQUIRE(v.input_present(1) && v.const_input(1), "%s: the %s input must be a constant initializer",
            v.op_type().c_str(), v.op_type() == "Reshape" ? "shape" : "axes");
  } else {
    REQUIRE(v.has_attr("axes"), "%s: axes attribute required", v.op_type().c_str());
  }
  if (v.op_type() == "Reshape") {
    REQUIRE(v.int_attr("allowzero", 0) == 0, "Reshape: allowzero=1 is not claimed");
    const auto target = const_ints(v.const_input(1));
    int unknown = 0;
    for (auto t : target) unknown += t == -1;
    REQUIRE(unknown <= 1, "Reshape: at most one -1 in the target shape");
  }
  return ClaimResult::yes();
}

// ---- PagedAttention: rust/src/ops/attention.rs:2748-2900 ------------------------------------
// The reference's checks for the forms this EP runs (separate K / V caches, causal, optional RoPE
// from structured cos / sin caches); slot_mapping, head_sink, q/k norms, rotary_offset and the
// LATENT layout are declined here (they stay with the next provider).
ClaimResult paged_claim(const NodeView& v) {
  REQUIRE(v.num_outputs() >= 1, "PagedAttention requires at least 1 output");
  const int o = out_dt(v, 0);
  REQUIRE(o == kF16 || o == kBF16, "PagedAttention is only supported for fp16/bf16 (T), got %s", dtype_name(o));
  const size_t nin = v.num_inputs();
  REQUIRE(nin >= 8 && nin <= 17, "expects 8 required inputs plus optional rotary inputs, got %zu", nin);
  REQUIRE(v.string_attr("kv_cache_layout", "SEPARATE") == "SEPARATE", "only the SEPARATE kv_cache_layout is implemented");
  for (size_t i : {0, 1, 2, 3, 4}) {
    REQUIRE(v.input_info(i), "input %zu (Q/K/V/cache) must be present with a float dtype", i);
    REQUIRE(in_dt(v, i) == o, "input %zu must share the output float dtype", i);
  }
  for (size_t i : {5, 6, 7}) {
    REQUIRE(v.input_info(i), "input %zu (positional) must be present", i);
    REQUIRE(in_dt(v, i) == kI32, "input %zu must be int32", i);
  }
  for (size_t i : {10, 11, 12, 13})
    REQUIRE(!v.input_present(i), "input %zu (slot_mapping / head_sink / q-k norm) is not implemented", i);
  const int64_t nh = v.int_attr("num_heads", 0), kvh = v.int_attr("kv_num_heads", 0);
  REQUIRE(nh > 0 && kvh > 0 && nh % kvh == 0, "num_heads (%lld) must be a positive multiple of kv_num_heads (%lld)",
          (long long)nh, (long long)kvh);
  auto* q = v.input_info(0);
  REQUIRE(q->shape.size() == 2 && q->shape[1] > 0 && q->shape[1] % nh == 0, "query must be [num_tokens,num_heads*head_size]");
  const int64_t head = q->shape[1] / nh;
  REQUIRE(head == 32 || head == 64 || head == 128, "head_size %lld is not 32, 64 or 128", (long long)head);
  const int64_t vh = v.int_attr("v_head_size", 0);
  REQUIRE(vh == 0 || vh == head, "v_head_size different from head_size is not implemented");
  REQUIRE(v.int_attr("rotary_offset", 0) == 0, "rotary_offset is not implemented");
  for (size_t i : {1, 2}) {
    auto* t = v.input_info(i);
    REQUIRE(t->shape.size() == 2 && t->shape[1] == kvh * head, "input %zu must be [num_tokens,kv_num_heads*head_size]", i);
  }
  for (size_t i : {3, 4}) {
    auto* t = v.input_info(i);
    REQUIRE(t->shape.size() == 4 && t->shape[1] > 0 && t->shape[2] == kvh && t->shape[3] == head,
            "input %zu must be [num_blocks,block_size,kv_num_heads,head_size] with a static block_size", i);
  }
  REQUIRE(v.int_attr("local_window_size", -1) == -1, "sliding-window attention (local_window_size) is not supported");
  REQUIRE(v.float_attr("softcap", 0.f) == 0.f, "attention softcap is not supported");
  for (size_t i = 1; i < v.num_outputs() && i < 3; ++i)
    if (v.output_present(i)) REQUIRE(out_dt(v, i) == o, "output %zu must share the output float dtype", i);
  if (v.int_attr("do_rotary", 0) != 0) {
    REQUIRE(v.input_present(8) && v.input_present(9), "do_rotary=1 requires cos_cache and sin_cache inputs");
    REQUIRE(in_dt(v, 8) == o && in_dt(v, 9) == o, "cos_cache/sin_cache must share the output float dtype");
    auto* c = v.input_info(8);
    REQUIRE(c->shape.size() == 2 && c->shape[1] > 0 && 2 * c->shape[1] <= head,
            "cos_cache must be [max_seq, rotary_dim/2] with rotary_dim <= head_size");
  }
  return ClaimResult::yes();
}

const OpEntry kTable[] = {
    {"com.microsoft", "MatMulNBits", -1, -1, OpKind::kMatMulNBits, matmulnbits_claim},
    {"com.microsoft", "GroupQueryAttention", -1, -1, OpKind::kGroupQueryAttention, gqa_claim},
    {"com.microsoft", "PagedAttention", -1, -1, OpKind::kPagedAttention, paged_claim},
    {"", "RMSNormalization", 23, -1, OpKind::kRmsNorm, rms_norm_claim},
    {"com.microsoft", "SimplifiedLayerNormalization", -1, -1, OpKind::kSimplifiedLayerNorm,
     simplified_layer_norm_claim},
    // Mis-stamped default-domain form that some exporters emit (norm.rs:938-952).
    {"", "SimplifiedLayerNormalization", -1, -1, OpKind::kSimplifiedLayerNorm, simplified_layer_norm_claim},
    {"com.microsoft", "SkipSimplifiedLayerNormalization", -1, -1, OpKind::kSkipSimplifiedLayerNorm,
     skip_rms_norm_claim},
    {"com.microsoft", "GatherBlockQuantized", -1, -1, OpKind::kGatherBlockQuantized, gbq_claim},
    {"", "Add", 7, -1, OpKind::kAdd, binary_claim},
    {"", "Sub", 7, -1, OpKind::kSub, binary_claim},
    {"", "Mul", 7, -1, OpKind::kMul, binary_claim},
    {"", "Sigmoid", 6, -1, OpKind::kSigmoid, sigmoid_claim},
    {"", "Cast", 6, -1, OpKind::kCast, cast_claim},
    {"", "Shape", 1, -1, OpKind::kShape, shape_claim},
    {"", "Gather", 1, -1, OpKind::kGather, gather_claim},
    {"", "ReduceSum", 1, -1, OpKind::kReduceSum, reduce_sum_claim},
    {"", "Unsqueeze", 1, -1, OpKind::kUnsqueeze, int_layout_claim},
    {"", "Squeeze", 1, -1, OpKind::kSqueeze, int_layout_claim},
    {"", "Reshape", 5, -1, OpKind::kReshape, int_layout_claim},
};

}  // namespace

bool is_ep_float(int dt) { return dt == kF32 || dt == kF16 || dt == kBF16; }

std::vector<int64_t> const_ints(const Initializer* init) {
  std::vector<int64_t> v;
  if (!init) return v;
  const int64_t n = init->numel();
  if (init->dtype == kI64 && init->bytes.size() == (size_t)n * 8) {
    v.resize(n);
    memcpy(v.data(), init->bytes.data(), (size_t)n * 8);
  } else if (init->dtype == kI32 && init->bytes.size() == (size_t)n * 4) {
    for (int64_t i = 0; i < n; ++i) {
      int32_t x;
      memcpy(&x, init->bytes.data() + 4 * i, 4);
      v.push_back(x);
    }
  }
  return v;
}

const char* op_kind_name(OpKind k) {
  switch (k) {
    case OpKind::kMatMulNBits: return "MatMulNBits";
    case OpKind::kGroupQueryAttention: return "GroupQueryAttention";
    case OpKind::kPagedAttention: return "PagedAttention";
    case OpKind::kRmsNorm: return "RMSNormalization";
    case OpKind::kSimplifiedLayerNorm: return "SimplifiedLayerNormalization";
    case OpKind::kSkipSimplifiedLayerNorm: return "SkipSimplifiedLayerNormalization";
    case OpKind::kGatherBlockQuantized: return "GatherBlockQuantized";
    case OpKind::kAdd: return "Add";
    case OpKind::kSub: return "Sub";
    case OpKind::kMul: return "Mul";
    case OpKind::kSigmoid: return "Sigmoid";
    case OpKind::kCast: return "Cast";
    case OpKind::kShape: return "Shape";
    case OpKind::kGather: return "Gather";
    case OpKind::kReduceSum: return "ReduceSum";
    case OpKind::kUnsqueeze: return "Unsqueeze";
    case OpKind::kSqueeze: return "Squeeze";
    case OpKind::kReshape: return "Reshape";
  }
  return "?";
}

const ValueInfo* NodeView::input_info(size_t i) const {
  if (!input_present(i)) return nullptr;
  const std::string& name = n_.inputs[i];
  if (auto* vi = g_.value(name)) return vi;
  if (auto* init = g_.initializer(name)) {
    tmp_.name = name;
    tmp_.dtype = init->dtype;
    tmp_.shape = init->shape;
    tmp_.has_shape = true;
    return &tmp_;
  }
  return nullptr;
}

const ValueInfo* NodeView::output_info(size_t i) const {
  if (!output_present(i)) return nullptr;
  return g_.value(n_.outputs[i]);
}

const Initializer* NodeView::const_input(size_t i) const {
  if (!input_present(i)) return nullptr;
  return g_.initializer(n_.inputs[i]);
}

std::string NodeView::string_attr(const std::string& k, const std::string& d) const {
  auto it = n_.attrs.find(k);
  return (it != n_.attrs.end() && it->second.kind == Attribute::kString) ? it->second.s : d;
}

const OpEntry* find_entry(const std::string& domain, const std::string& op_type, int ver) {
  const std::string dom = domain == "ai.onnx" ? "" : domain;
  for (const auto& e : kTable) {
    if (dom == e.domain && op_type == e.op_type && (e.min_opset < 0 || ver >= e.min_opset) &&
        (e.max_opset < 0 || ver <= e.max_opset))
      return &e;
  }
  return nullptr;
}

ClaimResult claim_decision(const NodeView& v) {
  const OpEntry* e = find_entry(v.domain(), v.op_type(), v.since_version());
  if (!e) {
    std::string where = v.domain().empty() ? "" : " (domain " + v.domain() + ")";
    return ClaimResult::no("no B200 handler for " + v.op_type() + where + " at opset " +
                           std::to_string(v.since_version()));
  }
  return e->claim(v);
}

}  // namespace b200ep
