// Op registry and claim predicates (reference: rust/src/registry.rs:16-217 for the
// (domain, op, opset-range) -> {handler, claim} table and the NodeView read helpers, and the
// per-op claims in rust/src/ops/{quant,attention,norm,elementwise}.rs).
#pragma once

#include <string>
#include <vector>

#include "graph.h"

namespace b200ep {

enum class OpKind {
  kMatMulNBits,
  kGroupQueryAttention,
  kPagedAttention,
  kRmsNorm,                // ai.onnx RMSNormalization (eps default 1e-6)
  kSimplifiedLayerNorm,    // com.microsoft / mis-stamped default domain (eps default 1e-5)
  kSkipSimplifiedLayerNorm,
  kGatherBlockQuantized,
  kAdd,
  kSub,
  kMul,
  kSigmoid,
  kCast,
  // integer glue of exported decoders (attention mask -> seqlens_k / total_sequence_length)
  kShape,
  kGather,
  kReduceSum,
  kUnsqueeze,
  kSqueeze,
  kReshape,
};

const char* op_kind_name(OpKind k);

// Claim-time read view of one node (the reference's NodeView): dtypes and shapes of inputs and
// outputs (initializers included), presence of optional slots, attributes.
class NodeView {
 public:
  NodeView(const Graph& g, const Node& n) : g_(g), n_(n) {}
  const Node& node() const { return n_; }
  const std::string& op_type() const { return n_.op_type; }
  const std::string& domain() const { return n_.domain; }
  int since_version() const { return g_.opset(n_.domain); }
  size_t num_inputs() const { return n_.inputs.size(); }
  size_t num_outputs() const { return n_.outputs.size(); }
  bool input_present(size_t i) const { return n_.input_present(i); }
  bool output_present(size_t i) const { return n_.output_present(i); }
  // nullptr when the slot is absent or carries no type information
  const ValueInfo* input_info(size_t i) const;
  const ValueInfo* output_info(size_t i) const;
  const Initializer* const_input(size_t i) const;
  int64_t int_attr(const std::string& k, int64_t d) const { return n_.int_attr(k, d); }
  bool has_attr(const std::string& k) const { return n_.has_attr(k); }
  std::vector<int64_t> ints_attr(const std::string& k) const { return n_.ints_attr(k); }
  float float_attr(const std::string& k, float d) const { return n_.float_attr(k, d); }
  std::string string_attr(const std::string& k, const std::string& d) const;

 private:
  const Graph& g_;
  const Node& n_;
  mutable ValueInfo tmp_;
};

struct ClaimResult {
  bool ok = true;
  std::string reason;  // why the node stays on CPU when !ok
  static ClaimResult yes() { return {}; }
  static ClaimResult no(std::string r) { return {false, std::move(r)}; }
};

struct OpEntry {
  const char* domain;
  const char* op_type;
  int min_opset;  // -1 = unbounded
  int max_opset;
  OpKind kind;
  ClaimResult (*claim)(const NodeView&);
};

const OpEntry* find_entry(const std::string& domain, const std::string& op_type, int since_version);
// The claim decision with its reason (the reference's claim_decision, registry.rs:175-192).
ClaimResult claim_decision(const NodeView& v);
inline bool claimable(const NodeView& v) { return claim_decision(v).ok; }

bool is_ep_float(int dtype);
inline bool is_ep_int(int dtype) { return dtype == 6 || dtype == 7; }  // int32 / int64
// Integer values of a constant int32 / int64 initializer (empty when it is neither).
std::vector<int64_t> const_ints(const Initializer* init);

}  // namespace b200ep
