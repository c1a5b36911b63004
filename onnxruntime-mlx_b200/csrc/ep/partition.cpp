#include "partition.h"

#include <algorithm>
#include <cstdlib>
#include <map>
#include <numeric>
#include <sstream>
#include <unordered_map>

#include "registry.h"

namespace b200ep {

namespace {

struct Adjacency {
  std::vector<std::vector<int>> succ, pred;
};

Adjacency adjacency(const Graph& g) {
  const int n = (int)g.nodes.size();
  std::unordered_map<std::string, int> producer;
  for (int i = 0; i < n; ++i)
    for (auto& o : g.nodes[i].outputs)
      if (!o.empty() && !producer.count(o)) producer[o] = i;
  Adjacency a;
  a.succ.assign(n, {});
  a.pred.assign(n, {});
  for (int j = 0; j < n; ++j) {
    std::vector<int> seen;
    for (auto& in : g.nodes[j].inputs) {
      if (in.empty()) continue;
      auto it = producer.find(in);
      if (it == producer.end() || it->second == j) continue;
      if (std::find(seen.begin(), seen.end(), it->second) != seen.end()) continue;
      seen.push_back(it->second);
      a.succ[it->second].push_back(j);
      a.pred[j].push_back(it->second);
    }
  }
  return a;
}

using Bits = std::vector<uint64_t>;
inline void bset(Bits& b, int i) { b[i >> 6] |= 1ull << (i & 63); }
inline bool btest(const Bits& b, int i) { return (b[i >> 6] >> (i & 63)) & 1; }
inline void bor(Bits& a, const Bits& b) {
  for (size_t i = 0; i < a.size(); ++i) a[i] |= b[i];
}
inline bool bintersects(const Bits& a, const Bits& b) {
  for (size_t i = 0; i < a.size(); ++i)
    if (a[i] & b[i]) return true;
  return false;
}

int uf_find(std::vector<int>& p, int x) {
  while (p[x] != x) {
    p[x] = p[p[x]];
    x = p[x];
  }
  return x;
}

}  // namespace

std::vector<std::vector<int>> build_convex_clusters(const Graph& g, const std::vector<bool>& supported) {
  const int n = (int)g.nodes.size();
  const size_t words = (n + 63) / 64;
  Adjacency adj = adjacency(g);

  // topological order (Kahn); a malformed cyclic graph falls back to index order
  std::vector<int> indeg(n), order;
  for (int i = 0; i < n; ++i) indeg[i] = (int)adj.pred[i].size();
  std::vector<int> stack;
  for (int i = 0; i < n; ++i)
    if (!indeg[i]) stack.push_back(i);
  while (!stack.empty()) {
    int u = stack.back();
    stack.pop_back();
    order.push_back(u);
    for (int v : adj.succ[u])
      if (--indeg[v] == 0) stack.push_back(v);
  }
  if ((int)order.size() != n) {
    order.resize(n);
    std::iota(order.begin(), order.end(), 0);
  }

  // reach[u]: every node reachable from u (excluding u)
  std::vector<Bits> reach(n, Bits(words, 0));
  for (auto it = order.rbegin(); it != order.rend(); ++it) {
    int u = *it;
    for (int v : adj.succ[u]) {
      bset(reach[u], v);
      bor(reach[u], reach[v]);
    }
  }

  std::vector<int> parent(n);
  std::iota(parent.begin(), parent.end(), 0);
  std::vector<Bits> members(n, Bits(words, 0)), creach(n, Bits(words, 0));
  for (int i = 0; i < n; ++i)
    if (supported[i]) {
      bset(members[i], i);
      creach[i] = reach[i];
    }
  std::vector<std::pair<int, int>> edges;
  for (int u = 0; u < n; ++u)
    if (supported[u])
      for (int v : adj.succ[u])
        if (supported[v]) edges.push_back({u, v});

  // S is convex iff no outside node x is both reachable from S and able to reach back into S.
  auto convex = [&](const Bits& s, const Bits& rs) {
    for (int x = 0; x < n; ++x) {
      if (btest(s, x) || !btest(rs, x)) continue;
      if (bintersects(reach[x], s)) return false;
    }
    return true;
  };

  bool changed = true;
  while (changed) {
    changed = false;
    for (auto [a, b] : edges) {
      int ra = uf_find(parent, a), rb = uf_find(parent, b);
      if (ra == rb) continue;
      Bits m = members[ra];
      bor(m, members[rb]);
      Bits r = creach[ra];
      bor(r, creach[rb]);
      if (!convex(m, r)) continue;
      parent[rb] = ra;
      members[ra] = std::move(m);
      creach[ra] = std::move(r);
      changed = true;
    }
  }

  std::map<int, std::vector<int>> grouped;
  for (int i = 0; i < n; ++i)
    if (supported[i]) grouped[uf_find(parent, i)].push_back(i);
  std::vector<std::vector<int>> clusters;
  for (auto& kv : grouped) clusters.push_back(kv.second);

  // Quotient acyclicity: two convex clusters may still form a cycle through unclaimed nodes;
  // contract and drop the smallest cluster on a cycle until the quotient graph is acyclic.
  for (;;) {
    std::vector<int> qid(n, -1);
    for (size_t c = 0; c < clusters.size(); ++c)
      for (int v : clusters[c]) qid[v] = (int)c;
    int next = (int)clusters.size();
    for (int& q : qid)
      if (q < 0) q = next++;
    std::vector<std::vector<int>> qs(next);
    std::vector<int> qin(next, 0);
    for (int u = 0; u < n; ++u)
      for (int v : adj.succ[u]) {
        int a = qid[u], b = qid[v];
        if (a != b && std::find(qs[a].begin(), qs[a].end(), b) == qs[a].end()) {
          qs[a].push_back(b);
          ++qin[b];
        }
      }
    std::vector<int> st;
    for (int i = 0; i < next; ++i)
      if (!qin[i]) st.push_back(i);
    int visited = 0;
    while (!st.empty()) {
      int u = st.back();
      st.pop_back();
      ++visited;
      for (int v : qs[u])
        if (--qin[v] == 0) st.push_back(v);
    }
    if (visited == next) break;
    int victim = -1;
    for (int i = 0; i < (int)clusters.size(); ++i)
      if (qin[i] > 0 && (victim < 0 || clusters[i].size() < clusters[victim].size())) victim = i;
    if (victim < 0) break;
    clusters.erase(clusters.begin() + victim);
  }
  for (auto& c : clusters) std::sort(c.begin(), c.end());
  std::sort(clusters.begin(), clusters.end(), [](auto& a, auto& b) { return a[0] < b[0]; });
  return clusters;
}

int select_layer_partition_span(const char* value, int layer_count) {
  if (!value) return 0;
  std::string v(value);
  v.erase(0, v.find_first_not_of(" \t"));
  v.erase(v.find_last_not_of(" \t") + 1);
  if (v == "0" || v == "off" || v == "false") return 0;
  if (v.empty() || v == "auto") {
    if (layer_count < 23) return 0;
    int span = (layer_count + 6) / 7;
    return std::min(8, std::max(4, span));
  }
  char* end = nullptr;
  long s = strtol(v.c_str(), &end, 10);
  if (end && *end == 0 && s > 0) return (int)s;
  return 0;
}

std::vector<int> infer_boundary_indices(const std::vector<std::string>& op_types,
                                        const std::vector<std::vector<int>>& successors,
                                        const std::vector<std::vector<int>>& predecessors,
                                        const std::vector<int>& anchors) {
  std::vector<int> out;
  if (anchors.size() < 2) return out;
  const int n = (int)op_types.size();
  for (size_t p = 0; p + 1 < anchors.size(); ++p) {
    const int cur = anchors[p], nxt = anchors[p + 1];
    std::vector<char> down(n, 0), up(n, 0);
    std::vector<int> st{cur};
    while (!st.empty()) {
      int u = st.back();
      st.pop_back();
      for (int s : successors[u])
        if (s <= nxt && !down[s]) {
          down[s] = 1;
          st.push_back(s);
        }
    }
    st = {nxt};
    while (!st.empty()) {
      int u = st.back();
      st.pop_back();
      for (int q : predecessors[u])
        if (q >= cur && !up[q]) {
          up[q] = 1;
          st.push_back(q);
        }
    }
    int found = -1;
    for (int i = nxt - 1; i > cur; --i)
      if (op_types[i] == "Add" && down[i] && up[i]) {
        found = i;
        break;
      }
    if (found < 0) return {};
    out.push_back(found);
  }
  return out;
}

static bool is_attention_anchor(const Node& n) {
  const bool present_cache = n.output_present(1) && n.output_present(2);
  if (n.domain == "com.microsoft" && n.op_type == "PagedAttention") return true;
  return present_cache && ((n.domain == "com.microsoft" &&
                            (n.op_type == "GroupQueryAttention" || n.op_type == "MultiHeadAttention")) ||
                           ((n.domain.empty() || n.domain == "ai.onnx") && n.op_type == "Attention"));
}

std::set<std::string> layer_boundary_outputs(const Graph& g, int* attention_layers) {
  std::set<std::string> out;
  int anchors_n = 0;
  for (auto& n : g.nodes) anchors_n += is_attention_anchor(n);
  if (attention_layers) *attention_layers = anchors_n;
  // model metadata wins (the reference's key, so exported models stay drop-in)
  for (const char* key : {"onnxruntime_ep_mlx.layer_boundary_outputs", "onnxruntime_ep_b200.layer_boundary_outputs"}) {
    auto it = g.metadata.find(key);
    if (it == g.metadata.end()) continue;
    std::stringstream ss(it->second);
    std::string tok;
    while (std::getline(ss, tok, ',')) {
      tok.erase(0, tok.find_first_not_of(" \t"));
      tok.erase(tok.find_last_not_of(" \t") + 1);
      if (!tok.empty()) out.insert(tok);
    }
    if (!out.empty()) return out;
  }
  Adjacency adj = adjacency(g);
  std::vector<std::string> ops;
  std::vector<int> anchors;
  for (int i = 0; i < (int)g.nodes.size(); ++i) {
    ops.push_back(g.nodes[i].op_type);
    if (is_attention_anchor(g.nodes[i])) anchors.push_back(i);
  }
  for (int idx : infer_boundary_indices(ops, adj.succ, adj.pred, anchors))
    if (!g.nodes[idx].outputs.empty() && !g.nodes[idx].outputs[0].empty()) out.insert(g.nodes[idx].outputs[0]);
  return out;
}

std::vector<std::vector<int>> split_layer_clusters(const Graph& g, std::vector<std::vector<int>> clusters,
                                                   const std::set<std::string>& boundary_outputs,
                                                   int layers_per_partition) {
  if (layers_per_partition <= 0 || boundary_outputs.empty()) return clusters;
  std::vector<std::vector<int>> split;
  for (auto& cl : clusters) {
    std::vector<int> part;
    int layers = 0;
    for (int idx : cl) {
      part.push_back(idx);
      bool end = false;
      for (auto& o : g.nodes[idx].outputs) end |= boundary_outputs.count(o) > 0;
      if (end && ++layers == layers_per_partition) {
        split.push_back(std::move(part));
        part.clear();
        layers = 0;
      }
    }
    if (!part.empty()) split.push_back(std::move(part));
  }
  return split;
}

CapabilityResult get_capability(const Graph& g, const char* layer_partition_setting) {
  CapabilityResult r;
  const int n = (int)g.nodes.size();
  std::vector<bool> supported(n, false);
  r.reasons.assign(n, "");
  for (int i = 0; i < n; ++i) {
    NodeView v(g, g.nodes[i]);
    ClaimResult c = claim_decision(v);
    supported[i] = c.ok;
    if (!c.ok) r.reasons[i] = c.reason;
  }
  auto clusters = build_convex_clusters(g, supported);
  int layers = 0;
  auto boundaries = layer_boundary_outputs(g, &layers);
  int span = select_layer_partition_span(layer_partition_setting, layers);
  r.groups = split_layer_clusters(g, std::move(clusters), boundaries, span);
  return r;
}

}  // namespace b200ep
