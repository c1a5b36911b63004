// extern "C" EP-core entry points (include/b200ep_ep.h).  Every entry catches exceptions and
// returns a status (the reference's FFI guard, rust/src/lib.rs:37-71).
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>

#include "../../../include/b200ep_ep.h"
#include "../common.cuh"
#include "../status.h"
#include "graph.h"
#include "partition.h"
#include "plan.h"
#include "registry.h"
#include "tp.h"

#ifdef B200EP_HAVE_NCCL
#include <nccl.h>
#endif

struct b200ep_graph {
  b200ep::Graph g;
};

struct b200ep_ep {
  b200ep::EpConfig cfg;
  std::string name = "B200ExecutionProvider";
  int device = 0;
  b200ep::CapabilityResult last;
  std::vector<std::vector<int>> groups;
};

struct b200ep_compiled {
  std::unique_ptr<b200ep::Plan> plan;
  std::string desc;
  int device = 0;
};

using namespace b200ep;

namespace {

#define GUARD_BEGIN try {
#define GUARD_END                                                                 \
  }                                                                               \
  catch (const std::exception& e) {                                               \
    return set_error(B200EP_EINTERNAL, std::string("exception: ") + e.what());    \
  }                                                                               \
  catch (...) {                                                                   \
    return set_error(B200EP_EINTERNAL, "unknown exception");                      \
  }

std::vector<int64_t> dims_of(int rank, const int64_t* dims) {
  std::vector<int64_t> v;
  for (int i = 0; i < rank; ++i) v.push_back(dims[i]);
  return v;
}

ValueInfo make_vi(const char* name, int dtype, int rank, const int64_t* dims) {
  ValueInfo vi;
  vi.name = name;
  vi.dtype = dtype;
  if (rank >= 0) {
    vi.shape = dims_of(rank, dims);
    vi.has_shape = true;
  }
  return vi;
}

Node* node_at(b200ep_graph* g, int i) {
  if (!g || i < 0 || i >= (int)g->g.nodes.size()) return nullptr;
  return &g->g.nodes[i];
}

void fill_args(const b200ep_tensor* t, size_t n, std::vector<TensorArg>& v);

std::vector<TensorArg> to_args(const b200ep_tensor* t, size_t n) {
  std::vector<TensorArg> v(n);
  fill_args(t, n, v);
  return v;
}

// the same into a caller-kept vector whose shape buffers are reused (no allocation per call in a
// decode loop)
void fill_args(const b200ep_tensor* t, size_t n, std::vector<TensorArg>& v) {
  v.resize(n);
  for (size_t i = 0; i < n; ++i) {
    v[i].data = t[i].data;
    v[i].dtype = t[i].dtype;
    v[i].shape.assign(t[i].dims, t[i].dims + std::max(0, (int)t[i].rank));
    v[i].on_device = t[i].on_device != 0;
  }
}

bool truthy(const char* v) { return v && *v && strcmp(v, "0") != 0 && strcmp(v, "false") != 0; }

}  // namespace

extern "C" {

B200EP_API b200ep_graph* b200ep_graph_create(void) {
  try {
    return new b200ep_graph();
  } catch (...) {
    return nullptr;
  }
}

B200EP_API void b200ep_graph_release(b200ep_graph* g) { delete g; }

B200EP_API int b200ep_graph_set_opset(b200ep_graph* g, const char* domain, int version) {
  GUARD_BEGIN
  B200EP_CHECK_ARG(g && domain, "graph/domain is null");
  g->g.opsets[strcmp(domain, "ai.onnx") == 0 ? "" : domain] = version;
  return B200EP_OK;
  GUARD_END
}

B200EP_API int b200ep_graph_add_value(b200ep_graph* g, const char* name, int dtype, int rank, const int64_t* dims) {
  GUARD_BEGIN
  B200EP_CHECK_ARG(g && name && rank <= B200EP_MAX_RANK && (rank <= 0 || dims), "bad value description");
  g->g.values[name] = make_vi(name, dtype, rank, dims);
  return B200EP_OK;
  GUARD_END
}

B200EP_API int b200ep_graph_add_input(b200ep_graph* g, const char* name, int dtype, int rank, const int64_t* dims) {
  GUARD_BEGIN
  B200EP_CHECK_ARG(g && name && rank <= B200EP_MAX_RANK && (rank <= 0 || dims), "bad input description");
  auto vi = make_vi(name, dtype, rank, dims);
  g->g.inputs.push_back(vi);
  g->g.values[name] = vi;
  return B200EP_OK;
  GUARD_END
}

B200EP_API int b200ep_graph_add_output(b200ep_graph* g, const char* name, int dtype, int rank, const int64_t* dims) {
  GUARD_BEGIN
  B200EP_CHECK_ARG(g && name && rank <= B200EP_MAX_RANK && (rank <= 0 || dims), "bad output description");
  auto vi = make_vi(name, dtype, rank, dims);
  g->g.outputs.push_back(vi);
  g->g.values[name] = vi;
  return B200EP_OK;
  GUARD_END
}

B200EP_API int b200ep_graph_add_initializer(b200ep_graph* g, const char* name, int dtype, int rank,
                                            const int64_t* dims, const void* data, size_t nbytes) {
  GUARD_BEGIN
  B200EP_CHECK_ARG(g && name && (nbytes == 0 || data) && rank <= B200EP_MAX_RANK, "bad initializer");
  auto init = std::make_shared<Initializer>();
  init->name = name;
  init->dtype = dtype;
  init->shape = dims_of(rank, dims);
  const int esz = dtype_size(dtype);
  B200EP_CHECK_ARG(esz > 0, "initializer dtype is not supported");
  B200EP_CHECK_ARG((int64_t)nbytes == init->numel() * esz, std::string("initializer ") + name + ": byte size mismatch");
  init->bytes.assign(static_cast<const uint8_t*>(data), static_cast<const uint8_t*>(data) + nbytes);
  g->g.initializers[name] = init;
  return B200EP_OK;
  GUARD_END
}

B200EP_API int b200ep_graph_add_node(b200ep_graph* g, const char* op_type, const char* domain, const char* name,
                                     int n_inputs, const char* const* inputs, int n_outputs,
                                     const char* const* outputs, int* node_index) {
  GUARD_BEGIN
  B200EP_CHECK_ARG(g && op_type && n_inputs >= 0 && n_outputs >= 0, "bad node description");
  Node n;
  n.op_type = op_type;
  n.domain = domain ? domain : "";
  if (n.domain == "ai.onnx") n.domain = "";
  n.name = name ? name : "";
  for (int i = 0; i < n_inputs; ++i) n.inputs.push_back(inputs[i] ? inputs[i] : "");
  for (int i = 0; i < n_outputs; ++i) n.outputs.push_back(outputs[i] ? outputs[i] : "");
  n.index = (int)g->g.nodes.size();
  g->g.nodes.push_back(std::move(n));
  if (node_index) *node_index = (int)g->g.nodes.size() - 1;
  return B200EP_OK;
  GUARD_END
}

B200EP_API int b200ep_graph_node_attr_int(b200ep_graph* g, int node, const char* name, int64_t value) {
  GUARD_BEGIN
  Node* n = node_at(g, node);
  B200EP_CHECK_ARG(n && name, "bad node index");
  Attribute a;
  a.kind = Attribute::kInt;
  a.i = value;
  n->attrs[name] = a;
  return B200EP_OK;
  GUARD_END
}

B200EP_API int b200ep_graph_node_attr_float(b200ep_graph* g, int node, const char* name, float value) {
  GUARD_BEGIN
  Node* n = node_at(g, node);
  B200EP_CHECK_ARG(n && name, "bad node index");
  Attribute a;
  a.kind = Attribute::kFloat;
  a.f = value;
  n->attrs[name] = a;
  return B200EP_OK;
  GUARD_END
}

B200EP_API int b200ep_graph_node_attr_string(b200ep_graph* g, int node, const char* name, const char* value) {
  GUARD_BEGIN
  Node* n = node_at(g, node);
  B200EP_CHECK_ARG(n && name && value, "bad node index");
  Attribute a;
  a.kind = Attribute::kString;
  a.s = value;
  n->attrs[name] = a;
  return B200EP_OK;
  GUARD_END
}

B200EP_API int b200ep_graph_node_attr_ints(b200ep_graph* g, int node, const char* name, const int64_t* v, int cnt) {
  GUARD_BEGIN
  Node* n = node_at(g, node);
  B200EP_CHECK_ARG(n && name && (cnt == 0 || v), "bad node index");
  Attribute a;
  a.kind = Attribute::kInts;
  a.ints.assign(v, v + cnt);
  n->attrs[name] = a;
  return B200EP_OK;
  GUARD_END
}

B200EP_API int b200ep_graph_set_metadata(b200ep_graph* g, const char* key, const char* value) {
  GUARD_BEGIN
  B200EP_CHECK_ARG(g && key && value, "bad metadata");
  g->g.metadata[key] = value;
  return B200EP_OK;
  GUARD_END
}

B200EP_API int b200ep_graph_num_nodes(const b200ep_graph* g) { return g ? (int)g->g.nodes.size() : 0; }

B200EP_API b200ep_ep* b200ep_ep_create(const char* const* keys, const char* const* values, size_t n) {
  try {
    auto* ep = new b200ep_ep();
    ep->cfg.summary = std::make_shared<SessionSummary>();
    ep->cfg.cuda_graph = !truthy(getenv("ONNXRUNTIME_EP_B200_NO_GRAPH"));
    ep->cfg.fuse = !truthy(getenv("ONNXRUNTIME_EP_B200_NO_FUSION"));
    ep->cfg.verbose = truthy(getenv("ONNXRUNTIME_EP_B200_VERBOSE"));
    if (const char* lp = getenv("ONNXRUNTIME_EP_B200_LAYER_PARTITIONS")) ep->cfg.layer_partitions = lp;
    if (const char* ta = getenv("ONNXRUNTIME_EP_B200_TP_ATTENTION"))
      ep->cfg.tp_replicate_attention = std::string(ta) == "replicated";
    for (size_t i = 0; i < n; ++i) {
      if (!keys || !values || !keys[i] || !values[i]) continue;
      std::string k = keys[i], v = values[i];
      if (k == "cuda_graph") ep->cfg.cuda_graph = truthy(v.c_str());
      else if (k == "fuse") ep->cfg.fuse = truthy(v.c_str());
      else if (k == "verbose") ep->cfg.verbose = truthy(v.c_str());
      else if (k == "layer_partitions") ep->cfg.layer_partitions = v;
      else if (k == "device_id") ep->device = atoi(v.c_str());
      else if (k == "registration_name") ep->name = v;
      else if (k == "tp_attention") ep->cfg.tp_replicate_attention = v == "replicated";
    }
    return ep;
  } catch (...) {
    return nullptr;
  }
}

B200EP_API void b200ep_ep_release(b200ep_ep* ep) {
  if (ep && ep->cfg.verbose && ep->cfg.summary) fprintf(stderr, "%s\n", ep->cfg.summary->text().c_str());
  delete ep;
}

B200EP_API int b200ep_ep_summary(const b200ep_ep* ep, char* out, size_t cap, size_t* needed) {
  GUARD_BEGIN
  B200EP_CHECK_ARG(ep && ep->cfg.summary, "ep is null");
  const std::string js = ep->cfg.summary->json();
  if (needed) *needed = js.size() + 1;
  if (out && cap > 0) {
    const size_t n = std::min(cap - 1, js.size());
    memcpy(out, js.data(), n);
    out[n] = 0;
  }
  return B200EP_OK;
  GUARD_END
}

B200EP_API const char* b200ep_ep_name(const b200ep_ep* ep) { return ep ? ep->name.c_str() : ""; }

B200EP_API int b200ep_ep_get_capability(b200ep_ep* ep, const b200ep_graph* g, int32_t* node_group,
                                        int32_t* num_groups) {
  GUARD_BEGIN
  B200EP_CHECK_ARG(ep && g, "ep/graph is null");
  const char* lp = ep->cfg.layer_partitions.empty() ? nullptr : ep->cfg.layer_partitions.c_str();
  ep->last = get_capability(g->g, lp);
  ep->groups = ep->last.groups;
  if (node_group)
    for (size_t i = 0; i < g->g.nodes.size(); ++i) node_group[i] = -1;
  for (size_t gi = 0; gi < ep->groups.size(); ++gi)
    for (int ni : ep->groups[gi])
      if (node_group) node_group[ni] = (int32_t)gi;
  if (num_groups) *num_groups = (int32_t)ep->groups.size();
  if (ep->cfg.summary) {
    SessionSummary& sm = *ep->cfg.summary;
    std::lock_guard<std::mutex> lk(sm.mu);
    ++sm.getcap_calls;
    sm.total_nodes += (int64_t)g->g.nodes.size();
    sm.partitions += (int64_t)ep->groups.size();
    for (auto& gr : ep->groups) sm.claimed_nodes += (int64_t)gr.size();
    for (size_t i = 0; i < ep->last.reasons.size(); ++i)
      if (!ep->last.reasons[i].empty()) {
        auto& r = sm.rejected[g->g.nodes[i].op_type];
        if (r.first++ == 0) r.second = ep->last.reasons[i];
      }
  }
  if (ep->cfg.verbose) {
    int claimed = 0;
    for (auto& gr : ep->groups) claimed += (int)gr.size();
    fprintf(stderr, "[b200ep] claimed %d/%zu nodes in %zu partitions\n", claimed, g->g.nodes.size(),
            ep->groups.size());
    for (size_t i = 0; i < ep->last.reasons.size(); ++i)
      if (!ep->last.reasons[i].empty())
        fprintf(stderr, "[b200ep] unclaimed %s (%s): %s\n", g->g.nodes[i].op_type.c_str(),
                g->g.nodes[i].name.c_str(), ep->last.reasons[i].c_str());
  }
  return B200EP_OK;
  GUARD_END
}

B200EP_API const char* b200ep_ep_claim_reason(const b200ep_ep* ep, int node) {
  if (!ep || node < 0 || node >= (int)ep->last.reasons.size()) return "";
  return ep->last.reasons[node].c_str();
}

B200EP_API int b200ep_ep_compile(b200ep_ep* ep, const b200ep_graph* g, int group, b200ep_compiled** out) {
  GUARD_BEGIN
  B200EP_CHECK_ARG(ep && g && out, "null argument");
  B200EP_CHECK_ARG(group >= 0 && group < (int)ep->groups.size(), "group index out of range (call get_capability first)");
  B200EP_CUDA_RET(cudaSetDevice(ep->device));
  std::string err;
  auto plan = Plan::compile(g->g, ep->groups[group], ep->cfg, &err);
  if (!plan) return set_error(B200EP_EUNSUPPORTED, "compile failed: " + err);
  auto* c = new b200ep_compiled();
  c->plan = std::move(plan);
  c->device = ep->device;
  *out = c;
  return B200EP_OK;
  GUARD_END
}

B200EP_API void b200ep_compiled_release(b200ep_compiled* c) { delete c; }

B200EP_API int b200ep_compiled_num_inputs(const b200ep_compiled* c) {
  return c ? (int)c->plan->input_names().size() : 0;
}
B200EP_API int b200ep_compiled_num_outputs(const b200ep_compiled* c) {
  return c ? (int)c->plan->output_names().size() : 0;
}
B200EP_API const char* b200ep_compiled_input_name(const b200ep_compiled* c, int i) {
  if (!c || i < 0 || i >= (int)c->plan->input_names().size()) return "";
  return c->plan->input_names()[i].c_str();
}
B200EP_API const char* b200ep_compiled_output_name(const b200ep_compiled* c, int i) {
  if (!c || i < 0 || i >= (int)c->plan->output_names().size()) return "";
  return c->plan->output_names()[i].c_str();
}

B200EP_API int b200ep_compiled_output_shapes(b200ep_compiled* c, const b200ep_tensor* inputs, size_t n_inputs,
                                             b200ep_tensor* outputs, size_t n_outputs) {
  GUARD_BEGIN
  B200EP_CHECK_ARG(c && (n_inputs == 0 || inputs) && (n_outputs == 0 || outputs), "null argument");
  B200EP_CHECK_ARG(n_outputs == c->plan->output_names().size(), "output count mismatch");
  std::vector<std::vector<int64_t>> shapes;
  int rc = c->plan->output_shapes(to_args(inputs, n_inputs), &shapes);
  if (rc) return rc;
  for (size_t i = 0; i < n_outputs; ++i) {
    B200EP_CHECK_ARG(shapes[i].size() <= B200EP_MAX_RANK, "output rank too large");
    outputs[i].dtype = c->plan->output_dtypes()[i];
    outputs[i].rank = (int32_t)shapes[i].size();
    for (size_t d = 0; d < shapes[i].size(); ++d) outputs[i].dims[d] = shapes[i][d];
  }
  return B200EP_OK;
  GUARD_END
}

B200EP_API int b200ep_compiled_run(b200ep_compiled* c, const b200ep_tensor* inputs, size_t n_inputs,
                                   b200ep_tensor* outputs, size_t n_outputs, void* stream) {
  GUARD_BEGIN
  B200EP_CHECK_ARG(c && (n_inputs == 0 || inputs) && (n_outputs == 0 || outputs), "null argument");
  B200EP_CUDA_RET(cudaSetDevice(c->device));
  static thread_local std::vector<TensorArg> ins, outs;
  fill_args(inputs, n_inputs, ins);
  fill_args(outputs, n_outputs, outs);
  return c->plan->run(ins, outs, static_cast<cudaStream_t>(stream));
  GUARD_END
}

B200EP_API const char* b200ep_compiled_describe(b200ep_compiled* c) {
  if (!c) return "";
  c->desc = c->plan->describe();
  return c->desc.c_str();
}

B200EP_API int b200ep_compiled_launches_per_run(const b200ep_compiled* c) {
  return c ? c->plan->launches_per_run() : 0;
}

B200EP_API int b200ep_tp_unique_id(void* out128) {
  GUARD_BEGIN
  B200EP_CHECK_ARG(out128, "null output");
#ifdef B200EP_HAVE_NCCL
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return set_error(B200EP_ENCCL, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
  memcpy(out128, &id, sizeof(id));
  return B200EP_OK;
#else
  return set_error(B200EP_EUNSUPPORTED, "library built without NCCL");
#endif
  GUARD_END
}

B200EP_API int b200ep_tp_shard_preview(const b200ep_graph* g, int rank, int world, char* out, size_t cap,
                                      size_t* needed) {
  GUARD_BEGIN
  B200EP_CHECK_ARG(g && world >= 1 && rank >= 0 && rank < world, "bad graph or rank/world");
  b200ep::EpConfig cfg;
  cfg.host_only = true;
  if (world > 1) {
    cfg.tp = std::make_shared<TpContext>();
    cfg.tp->rank = rank;
    cfg.tp->world = world;
  }
  std::vector<int> nodes(g->g.nodes.size());
  for (size_t i = 0; i < nodes.size(); ++i) nodes[i] = (int)i;
  std::string err;
  auto plan = Plan::compile(g->g, nodes, cfg, &err);
  if (!plan) return set_error(B200EP_EUNSUPPORTED, "shard preview failed: " + err);
  const std::string js = plan->preview();
  if (needed) *needed = js.size() + 1;
  if (out && cap > 0) {
    const size_t n = std::min(cap - 1, js.size());
    memcpy(out, js.data(), n);
    out[n] = 0;
  }
  return B200EP_OK;
  GUARD_END
}

B200EP_API int b200ep_ep_set_tensor_parallel(b200ep_ep* ep, int rank, int world, const void* nccl_unique_id) {
  GUARD_BEGIN
  B200EP_CHECK_ARG(ep && world >= 1 && rank >= 0 && rank < world, "bad tensor-parallel rank/world");
  if (world == 1) {
    ep->cfg.tp.reset();
    return B200EP_OK;
  }
  B200EP_CHECK_ARG(nccl_unique_id, "null NCCL unique id");
#ifdef B200EP_HAVE_NCCL
  B200EP_CUDA_RET(cudaSetDevice(ep->device));
  ncclUniqueId id;
  memcpy(&id, nccl_unique_id, sizeof(id));
  ncclComm_t comm = nullptr;
  ncclResult_t r = ncclCommInitRank(&comm, world, id, rank);
  if (r != ncclSuccess) return set_error(B200EP_ENCCL, std::string("ncclCommInitRank: ") + ncclGetErrorString(r));
  auto tp = std::make_shared<TpContext>();
  tp->rank = rank;
  tp->world = world;
  tp->comm = comm;
  tp->owns_comm = true;
  // decode-sized partial sums (16 rows x 16384 fp16/bf16 per source rank) travel through the
  // peer mailboxes; larger ones through NCCL
  if (!truthy(getenv("ONNXRUNTIME_EP_B200_NO_PEER_ALLREDUCE")))
    if (int rc = tp_mailbox_init(*tp, (size_t)16 * 16384 * 2)) return rc;
  ep->cfg.tp = tp;
  return B200EP_OK;
#else
  return set_error(B200EP_EUNSUPPORTED, "library built without NCCL");
#endif
  GUARD_END
}

}  // extern "C"
