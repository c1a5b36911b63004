// Graph IR the EP core works on.  It holds what the reference reads from ORT's graph API
// through NodeView (rust/src/registry.rs:240-1052) and copies into its plan
// (rust/src/engine.rs:12-162): value infos, initializers (owned host bytes), nodes with
// attributes, graph inputs/outputs and model metadata.  The mock host builds it through the
// b200ep_graph_* C ABI; an ORT shim fills it from OrtGraph.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace b200ep {

struct ValueInfo {
  std::string name;
  int dtype = 0;                 // ONNX element type; 0 = unknown
  std::vector<int64_t> shape;    // -1 = symbolic dimension
  bool has_shape = false;
};

struct Initializer {
  std::string name;
  int dtype = 0;
  std::vector<int64_t> shape;
  std::vector<uint8_t> bytes;    // owned copy (the reference copies initializer bytes: ep.rs:1213-1298)
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
};

struct Attribute {
  enum Kind { kInt, kFloat, kString, kInts, kFloats } kind = kInt;
  int64_t i = 0;
  float f = 0.f;
  std::string s;
  std::vector<int64_t> ints;
  std::vector<float> floats;
};

struct Node {
  std::string name, op_type, domain;
  std::vector<std::string> inputs;   // "" = absent optional input
  std::vector<std::string> outputs;  // "" = absent optional output
  std::map<std::string, Attribute> attrs;
  int index = -1;                    // position in Graph::nodes

  int64_t int_attr(const std::string& k, int64_t dflt) const {
    auto it = attrs.find(k);
    return (it != attrs.end() && it->second.kind == Attribute::kInt) ? it->second.i : dflt;
  }
  bool has_attr(const std::string& k) const { return attrs.count(k) != 0; }
  std::vector<int64_t> ints_attr(const std::string& k) const {
    auto it = attrs.find(k);
    if (it == attrs.end()) return {};
    if (it->second.kind == Attribute::kInts) return it->second.ints;
    if (it->second.kind == Attribute::kInt) return {it->second.i};
    return {};
  }
  float float_attr(const std::string& k, float dflt) const {
    auto it = attrs.find(k);
    if (it == attrs.end()) return dflt;
    if (it->second.kind == Attribute::kFloat) return it->second.f;
    if (it->second.kind == Attribute::kInt) return (float)it->second.i;
    return dflt;
  }
  bool input_present(size_t i) const { return i < inputs.size() && !inputs[i].empty(); }
  bool output_present(size_t i) const { return i < outputs.size() && !outputs[i].empty(); }
};

struct Graph {
  std::vector<ValueInfo> inputs;     // graph inputs (runtime-fed)
  std::vector<ValueInfo> outputs;    // graph outputs
  std::map<std::string, ValueInfo> values;  // every typed value (inputs, outputs, intermediates)
  std::map<std::string, std::shared_ptr<Initializer>> initializers;
  std::vector<Node> nodes;
  std::map<std::string, std::string> metadata;
  std::map<std::string, int> opsets;  // domain -> opset version ("" = ai.onnx)

  const ValueInfo* value(const std::string& name) const {
    auto it = values.find(name);
    return it == values.end() ? nullptr : &it->second;
  }
  const Initializer* initializer(const std::string& name) const {
    auto it = initializers.find(name);
    return it == initializers.end() ? nullptr : it->second.get();
  }
  int opset(const std::string& domain) const {
    auto it = opsets.find(domain == "ai.onnx" ? "" : domain);
    return it == opsets.end() ? (domain.empty() ? 21 : 1) : it->second;
  }
  bool is_graph_output(const std::string& name) const {
    for (auto& o : outputs)
      if (o.name == name) return true;
    return false;
  }
};

}  // namespace b200ep
