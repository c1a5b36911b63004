// GetCapability: claimed nodes -> maximal convex clusters -> layer partitions.
// Reference: build_convex_clusters (rust/src/ep.rs:691-895), infer_layer_boundary_outputs /
// infer_boundary_indices (ep.rs:372-483), select_layer_partition_span (ep.rs:359-370),
// split_annotated_layer_clusters (ep.rs:485-516), get_capability_impl (ep.rs:132-357).
#pragma once

#include <set>
#include <string>
#include <vector>

#include "graph.h"

namespace b200ep {

struct CapabilityResult {
  std::vector<std::vector<int>> groups;  // node indices per fused node, topological order inside
  std::vector<std::string> reasons;      // per node: "" when claimed, else why it stays on CPU
};

// Maximal convex clusters of the supported nodes (plus the quotient-acyclicity guard).
std::vector<std::vector<int>> build_convex_clusters(const Graph& g, const std::vector<bool>& supported);

// Layer span for a decoder with `layer_count` attention layers.  `value` is the
// ONNXRUNTIME_EP_B200_LAYER_PARTITIONS setting (nullptr = unset): "0"/"off"/"false" -> no split,
// "auto" -> the reference's heuristic, an integer -> that span.  Unset means no split on this EP
// (a CUDA graph per partition has no trace cost to bound); returns 0 for "no split".
int select_layer_partition_span(const char* value, int layer_count);

// Indices (into op_types) of the residual Add that closes each layer between consecutive
// attention anchors; empty when any layer has none.
std::vector<int> infer_boundary_indices(const std::vector<std::string>& op_types,
                                        const std::vector<std::vector<int>>& successors,
                                        const std::vector<std::vector<int>>& predecessors,
                                        const std::vector<int>& anchors);

std::set<std::string> layer_boundary_outputs(const Graph& g, int* attention_layers);

std::vector<std::vector<int>> split_layer_clusters(const Graph& g, std::vector<std::vector<int>> clusters,
                                                   const std::set<std::string>& boundary_outputs,
                                                   int layers_per_partition);

CapabilityResult get_capability(const Graph& g, const char* layer_partition_setting);

}  // namespace b200ep
