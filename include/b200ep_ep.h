/*
 * b200ep_ep.h — execution-provider core C ABI of the B200 int4 decode EP.
 *
 * This is the host side the reference implements in Rust behind ONNX Runtime's plugin-EP ABI
 * (rust/src/lib.rs, factory.rs, ep.rs, engine.rs, compiled.rs): a graph is described, the EP
 * claims the nodes it can run (GetCapability), each fused partition is compiled into a device
 * plan (Compile), and the plan runs once per call (Compute).  An ORT shim maps OrtGraph /
 * OrtKernelContext onto these calls; test harnesses and benchmarks call them directly.
 *
 * Conventions: see b200ep.h (ONNX element-type codes, B200EP_* status, b200ep_last_error).
 */
#ifndef B200EP_EP_H_
#define B200EP_EP_H_

#include <stddef.h>
#include <stdint.h>

#include "b200ep.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b200ep_graph b200ep_graph;
typedef struct b200ep_ep b200ep_ep;
typedef struct b200ep_compiled b200ep_compiled;

#define B200EP_MAX_RANK 8

/* A boundary tensor handed to b200ep_compiled_run.  on_device != 0: `data` is a device pointer
 * used in place; 0: host memory, staged to/from the device by the EP (the plugin's data
 * transfer; replaces the reference's null data-transfer stub, rust/src/factory.rs:221-253). */
typedef struct b200ep_tensor {
  void* data;
  int32_t dtype;
  int32_t rank;
  int64_t dims[B200EP_MAX_RANK];
  int32_t on_device;
} b200ep_tensor;

/* Graph description (replaces the reads the reference makes through ORT's graph API and
 * NodeView, rust/src/registry.rs:240-1052; initializer bytes are copied like ep.rs:1213-1298). */
B200EP_API b200ep_graph* b200ep_graph_create(void);
B200EP_API void b200ep_graph_release(b200ep_graph* g);
B200EP_API int b200ep_graph_set_opset(b200ep_graph* g, const char* domain, int version);
B200EP_API int b200ep_graph_add_value(b200ep_graph* g, const char* name, int dtype, int rank, const int64_t* dims);
B200EP_API int b200ep_graph_add_input(b200ep_graph* g, const char* name, int dtype, int rank, const int64_t* dims);
B200EP_API int b200ep_graph_add_output(b200ep_graph* g, const char* name, int dtype, int rank, const int64_t* dims);
B200EP_API int b200ep_graph_add_initializer(b200ep_graph* g, const char* name, int dtype, int rank,
                                            const int64_t* dims, const void* data, size_t nbytes);
/* Appends a node; "" in inputs/outputs marks an absent optional slot.  *node_index receives
 * its index (nodes must be added in topological order). */
B200EP_API int b200ep_graph_add_node(b200ep_graph* g, const char* op_type, const char* domain, const char* name,
                                     int n_inputs, const char* const* inputs, int n_outputs,
                                     const char* const* outputs, int* node_index);
B200EP_API int b200ep_graph_node_attr_int(b200ep_graph* g, int node, const char* name, int64_t value);
B200EP_API int b200ep_graph_node_attr_float(b200ep_graph* g, int node, const char* name, float value);
B200EP_API int b200ep_graph_node_attr_string(b200ep_graph* g, int node, const char* name, const char* value);
B200EP_API int b200ep_graph_node_attr_ints(b200ep_graph* g, int node, const char* name, const int64_t* v, int n);
B200EP_API int b200ep_graph_set_metadata(b200ep_graph* g, const char* key, const char* value);
B200EP_API int b200ep_graph_num_nodes(const b200ep_graph* g);

/* EP instance.  Options (key/value strings; the reference ignores session options,
 * factory.rs:191-199, and reads environment variables — both are honoured here):
 *   "cuda_graph" = "0"/"1", "fuse" = "0"/"1", "layer_partitions" = "off"/"auto"/<span>,
 *   "device_id" = <int>, "verbose" = "0"/"1".
 * Environment: ONNXRUNTIME_EP_B200_{NO_GRAPH, NO_FUSION, LAYER_PARTITIONS, VERBOSE}. */
B200EP_API b200ep_ep* b200ep_ep_create(const char* const* keys, const char* const* values, size_t n);
B200EP_API void b200ep_ep_release(b200ep_ep* ep);
B200EP_API const char* b200ep_ep_name(const b200ep_ep* ep);

/* GetCapability (get_capability_impl, rust/src/ep.rs:132-357): node_group[i] receives the fused
 * partition of node i or -1 when it stays on the CPU EP; *num_groups the partition count. */
B200EP_API int b200ep_ep_get_capability(b200ep_ep* ep, const b200ep_graph* g, int32_t* node_group,
                                        int32_t* num_groups);
/* Why node i was not claimed ("" when claimed) — from the last get_capability on this EP. */
B200EP_API const char* b200ep_ep_claim_reason(const b200ep_ep* ep, int node);

/* Compile (compile_impl / build_plan, rust/src/ep.rs:928-1211): weights are uploaded to HBM here. */
B200EP_API int b200ep_ep_compile(b200ep_ep* ep, const b200ep_graph* g, int group, b200ep_compiled** out);
B200EP_API void b200ep_compiled_release(b200ep_compiled* c);
B200EP_API int b200ep_compiled_num_inputs(const b200ep_compiled* c);
B200EP_API int b200ep_compiled_num_outputs(const b200ep_compiled* c);
B200EP_API const char* b200ep_compiled_input_name(const b200ep_compiled* c, int i);
B200EP_API const char* b200ep_compiled_output_name(const b200ep_compiled* c, int i);
/* Output dtypes and shapes for the given inputs (dims/rank/dtype of outputs[] are filled). */
B200EP_API int b200ep_compiled_output_shapes(b200ep_compiled* c, const b200ep_tensor* inputs, size_t n_inputs,
                                             b200ep_tensor* outputs, size_t n_outputs);
/* Compute (compute_impl, rust/src/ep.rs:1940-2134).  Ordered on `stream` (cudaStream_t). */
B200EP_API int b200ep_compiled_run(b200ep_compiled* c, const b200ep_tensor* inputs, size_t n_inputs,
                                   b200ep_tensor* outputs, size_t n_outputs, void* stream);
/* JSON summary: fused steps, weight bytes, runs, CUDA-graph captures/replays. */
B200EP_API const char* b200ep_compiled_describe(b200ep_compiled* c);
B200EP_API int b200ep_compiled_launches_per_run(const b200ep_compiled* c);

/* Host-only preview of the tensor-parallel plan of `rank` of `world` for the whole graph: lowers,
 * fuses and shards (no device memory, no NCCL) and writes a JSON array describing every step —
 * MatMulNBits geometry with FNV-1a hashes of the sliced weight initializers, attention heads, and
 * the inserted AllReduce / AllGather steps in launch order.  No counterpart in the reference (which
 * has no multi-GPU path); it lets the sharding be checked on a machine without GPUs.  *needed
 * receives the JSON length + 1; out may be NULL to query it. */
/* Session summary as JSON (reference: MlxTracer::log_summary, rust/src/trace.rs:640-735): claimed
 * / total nodes and per op type why nodes stayed on CPU, partitions compiled (time, weight bytes),
 * runs per path (decode / prefill / general) and how they ran (graph replay, capture, eager),
 * shape-key cache hits, host boundary bytes staged, host time in runs.  Same two-call sizing as
 * b200ep_tp_shard_preview.  With ONNXRUNTIME_EP_B200_VERBOSE=1 (or provider option verbose=1) the
 * text form is printed to stderr by b200ep_ep_release, as the reference does with
 * ONNXRUNTIME_EP_MLX_VERBOSE. */
B200EP_API int b200ep_ep_summary(const b200ep_ep* ep, char* out, size_t cap, size_t* needed);

B200EP_API int b200ep_tp_shard_preview(const b200ep_graph* g, int rank, int world, char* out, size_t cap,
                                      size_t* needed);

/* Tensor parallelism: attach this process (rank of world, one GPU each) to a communicator before
 * compiling; `nccl_unique_id` is the 128-byte ncclUniqueId rank 0 created
 * (b200ep_tp_unique_id) and broadcast.  Compiled plans then shard column-/row-parallel. */
B200EP_API int b200ep_tp_unique_id(void* out128);
B200EP_API int b200ep_ep_set_tensor_parallel(b200ep_ep* ep, int rank, int world, const void* nccl_unique_id);

#ifdef __cplusplus
}
#endif

#endif /* B200EP_EP_H_ */
