// Compiled partition ("plan"): the B200 counterpart of the reference's Plan + compiled closures
// (rust/src/engine.rs:409-573, rust/src/compiled.rs:503-1203).
//
// compile():  lowers the partition's nodes to device steps, uploads the initializers the steps
//             read (weights stay resident in HBM), and runs the fusion passes
//               - q/k/v MatMulNBits sharing one input -> one GEMV writing packed QKV, consumed by
//                 GroupQueryAttention in its packed form;
//               - gate/up MatMulNBits + Sigmoid/Mul/Mul (SwiGLU) -> one GEMV + one fused SiLU*up;
//               - (Skip)SimplifiedLayerNorm or SiLU*up whose only consumer is a prepacked GEMV ->
//                 folded into that GEMV's activation staging (decode-sized rows).
// run():      binds the boundary tensors (device pointers in place; host tensors staged), infers
//             the shapes of the step, allocates per-shape-key buffers once, and launches the
//             steps.  With CUDA graphs on, the launches of a (shape key, boundary pointers) pair
//             are captured once and replayed; decode positions come from device-side seqlens_k,
//             so one graph serves every token of a decode loop.
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "graph.h"
#include "registry.h"

namespace b200ep {

struct TpContext;  // tensor-parallel communicator (tp.h)

// Session digest of one EP (reference: MlxTracer::log_summary, rust/src/trace.rs:640-735, printed
// when ONNXRUNTIME_EP_MLX_VERBOSE is set): claim rate and why nodes stayed on CPU, compiled
// partitions, runs per path and shape-key cache, boundary copies, host time.  Shared by the EP and
// its compiled partitions; printed to stderr when the EP is released with
// ONNXRUNTIME_EP_B200_VERBOSE=1, and returned as JSON by b200ep_ep_summary.
struct SessionSummary {
  mutable std::mutex mu;
  int64_t getcap_calls = 0, total_nodes = 0, claimed_nodes = 0, partitions = 0;
  std::map<std::string, std::pair<int64_t, std::string>> rejected;  // op type -> (nodes, first reason)
  int64_t compiles = 0, weight_bytes = 0;
  double compile_ms = 0;
  // runs by path: decode (every attention step has one query row), prefill (more rows), general
  // (no attention); how they executed: CUDA-graph replay, graph capture, eager
  int64_t path_decode = 0, path_prefill = 0, path_general = 0;
  int64_t graph_replays = 0, graph_captures = 0, eager_runs = 0;
  int64_t key_hits = 0, key_misses = 0;  // per-shape-key program cache
  int64_t h2d_bytes = 0, d2h_bytes = 0;  // host boundary tensors staged through the EP
  double run_ms = 0;                     // host time inside compiled runs
  std::string json() const;
  std::string text() const;
};

struct EpConfig {
  bool cuda_graph = true;
  bool fuse = true;
  bool verbose = false;
  std::string layer_partitions;  // "" = unset
  std::shared_ptr<TpContext> tp;  // null = single GPU
  // tensor parallel: attention (q/k/v, GroupQueryAttention, o_proj) on every rank in full instead of
  // sharded by KV head, so the only all-reduce of a layer is the FFN's at the layer boundary
  // (provider option tp_attention = "replicated"; default "sharded")
  bool tp_replicate_attention = false;
  bool host_only = false;         // lower, fuse and shard on the host only (no upload): preview()
  std::shared_ptr<SessionSummary> summary;  // null = not recorded
};

struct TensorArg {
  void* data = nullptr;
  int dtype = 0;
  std::vector<int64_t> shape;
  bool on_device = true;
};

struct DevMem {
  void* p = nullptr;
  size_t bytes = 0;
  DevMem() = default;
  DevMem(const DevMem&) = delete;
  DevMem& operator=(const DevMem&) = delete;
  ~DevMem();
  int alloc(size_t n);
};

struct Slot {
  enum Kind { kTemp, kInput, kOutput, kConst } kind = kTemp;
  std::string name;
  int dtype = 0;
  int io = -1;  // boundary index for inputs / outputs
  std::shared_ptr<DevMem> cmem;       // constants
  std::vector<int64_t> cshape;        // constants
  std::vector<uint8_t> host_copy;     // constants small enough to read on the host
  // per run
  std::vector<int64_t> shape;
  void* ptr = nullptr;
  // integer values known on the host (int constants, Shape results, host-resident scalars and
  // what the integer glue computes from them); such values are uploaded, not computed by kernels
  bool hknown = false;
  std::vector<int64_t> hval;
  // inputs whose extent along a key axis changes every call without changing the program: the
  // call's real shape (shape then holds the program's capacity)
  std::vector<int64_t> rshape;
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
};

enum class StepKind {
  kMnb, kGqa, kRms, kBinary, kSigmoid, kSiluMul, kCast, kGbq, kAllReduce, kAllGather, kPaged,
  // integer glue: Shape, Gather of a shape vector, ReduceSum over the last axis, and the
  // value-preserving Unsqueeze / Squeeze / Reshape (kCopy)
  kShape, kGatherIdx, kReduceSum, kCopy
};

struct Step {
  StepKind kind;
  std::string name;   // originating node(s)
  std::vector<int> in, out;
  // MatMulNBits
  int64_t K = 0, N = 0;
  int bits = 4, block = 32;
  int wB = -1, wS = -1, wZ = -1;
  // norms
  float eps = 1e-5f;
  bool skip = false;
  // GroupQueryAttention
  int num_heads = 0, kv_heads = 0, head_size = 0;
  bool packed = false;
  int do_rotary = 1, interleaved = 0, local_window = -1;
  bool sliding = false;  // sliding_window_cache = 1: the cache reclaims rows (gqa_sliding.cu)
  float scale = 0.f, qk_eps = 1e-6f;
  int ws_slot = -1;  // workspace (temp, zero-filled when allocated)
  // binary
  int bop = 0;
  // cast
  int to = 0;
  // GatherBlockQuantized
  int64_t gbq_rows = 0, gbq_dim = 0;
  // tensor parallel gather: shard width along the last axis
  int64_t shard_cols = 0;
  // integer glue: Shape's [start, end) (unnormalised attributes); ReduceSum keepdims; Gather's
  // constant indices and their rank; Unsqueeze / Squeeze axes or the Reshape target (layout 1 / 2 / 3)
  int64_t shp_start = 0, shp_end = INT64_MAX;
  bool keepdims = true;
  std::vector<int64_t> ivals;
  int idx_rank = 0, layout = 0;
  // MatMulNBits weights prepacked for the tensor-core path (fp16/bf16, int4)
  bool prepacked = false;
  // fused gate/up whose weight rows are interleaved 8 gate / 8 up per 16-row tile: the step writes
  // SiLU(gate) * up (N / 2 columns); paths that cannot (the GEMM, the SIMT kernel) write both into
  // ws_slot and a separate kernel applies it
  bool swiglu = false;
  std::shared_ptr<DevMem> pk_w;
  // producer of in[0] folded into the GEMV's activation staging (MnbProKind); the standalone
  // producer still runs into in[0] when the rows do not fit the staging area
  int pro = 0;
  int pro_x = -1, pro_skip = -1, pro_gamma = -1, pro_res = -1;
  float pro_eps = 0.f;
  int64_t pro_n = 0;  // SiLU*up: width of the gate (= K)
  // tensor parallel, decode sizes: the all-reduce between a row-parallel GEMV (ar_out) and the
  // GEMV whose skip-norm prologue reads its sum (pro_ar) runs through the peer mailboxes; the
  // AllReduce step between them (ar_skip) then launches nothing
  bool ar_out = false, pro_ar = false, ar_skip = false;
  int ar_block = 0;  // block size of the consuming GEMV (its staging decides the fused path)
};

struct PlanStats {
  int nodes = 0, steps = 0, fused_qkv = 0, fused_swiglu = 0, fused_norm = 0, fused_act = 0, swiglu_epilogue = 0;
  int64_t weight_bytes = 0;
  int64_t runs = 0, graph_replays = 0, graph_captures = 0;
  int peer_allreduce = 0;
};

class Plan {
 public:
  static std::unique_ptr<Plan> compile(const Graph& g, const std::vector<int>& nodes, const EpConfig& cfg,
                                       std::string* err);
  ~Plan();
  const std::vector<std::string>& input_names() const { return in_names_; }
  const std::vector<std::string>& output_names() const { return out_names_; }
  const std::vector<int>& output_dtypes() const { return out_dtypes_; }
  // Output shapes for the given inputs (host reads only of host-resident scalar inputs).
  int output_shapes(const std::vector<TensorArg>& in, std::vector<std::vector<int64_t>>* shapes);
  int run(const std::vector<TensorArg>& in, const std::vector<TensorArg>& out, cudaStream_t st);
  std::string describe() const;
  // Host-side view of the compiled steps (host_only plans): per step its kind, name and geometry,
  // and for MatMulNBits a 64-bit FNV-1a hash of each (sliced) weight initializer.
  std::string preview() const;
  const PlanStats& stats() const { return stats_; }
  // number of device kernels one run launches (for the launch-count claim of the bench)
  int launches_per_run() const;

 private:
  struct Program;  // per-shape-key buffers and captured graphs
  Plan() = default;
  static std::unique_ptr<Plan> compile_impl(const Graph& g, const std::vector<int>& nodes, const EpConfig& cfg,
                                            std::string* err);
  int lower(const Graph& g, const std::vector<int>& nodes, std::string* err);
  int upload_constants(const Graph& g, std::string* err);
  void fuse_qkv();
  void fuse_swiglu();
  void fuse_prologues();
  void fuse_peer_allreduce();
  void fuse_swiglu_epilogue();
  bool ar_fused(int64_t M, int64_t hidden, int cons_block) const;
  int shard_for_tp(std::string* err);
  int infer(std::vector<Slot>& slots, std::string* err) const;
  // integer glue on the host: output shape of a glue step, and its values when every input's
  // values are known (returns non-zero with err set on an invalid index / shape)
  int infer_glue(const Step& st, std::vector<Slot>& S, std::string* err) const;
  // per call, before the launches: copy inputs with a changing key axis into the program's
  // buffers, re-evaluate the host-side glue for this call's shapes and upload its values
  int stage_dynamic(Program& prog, const std::vector<TensorArg>& in, cudaStream_t st);
  // how an input enters the program key: 0 as is; 1 only its rank (the input feeds only Shape);
  // 2 its last axis as a power-of-two capacity (it feeds only Shape and ReduceSum over that axis)
  void compute_free_rules();
  std::vector<int64_t> key_shape(int io, const std::vector<int64_t>& shape) const;
  int launch_steps(const std::vector<Slot>& slots, Program& prog, cudaStream_t st);
  int run_locked(const std::vector<TensorArg>& in, const std::vector<TensorArg>& out, cudaStream_t st);
  int slot_of(const std::string& name);

  EpConfig cfg_;
  std::vector<Slot> slots_;
  std::map<std::string, int> slot_index_;
  std::vector<Step> steps_;
  std::vector<std::string> in_names_, out_names_;
  std::vector<int> free_rule_;  // per boundary input (compute_free_rules)
  std::vector<int> out_dtypes_;
  std::map<std::string, std::unique_ptr<Program>> programs_;
  std::mutex mu_;
  PlanStats stats_;
  cudaStream_t stream_ = nullptr;
  cudaEvent_t ev_in_ = nullptr, ev_out_ = nullptr;
  // repeated calls with the same boundary tensors (a decode loop): the signature (pointer,
  // residency, shape of every boundary tensor) of the last call, its program and graph
  std::vector<int64_t> last_sig_;
  Program* last_prog_ = nullptr;
  cudaGraphExec_t last_exec_ = nullptr;
  // host-side constant data used while lowering / fusing (weights before upload)
  std::map<int, std::shared_ptr<Initializer>> pending_consts_;
  // ONNXRUNTIME_EP_B200_PROFILE: per-step CUDA-event times of eager runs (no graph), printed on
  // destruction as totals per step name (steps run serialised, so PDL overlap is not included)
  bool prof_ = false;
  std::vector<cudaEvent_t> prof_ev_;
  std::map<std::string, std::pair<int64_t, double>> prof_ms_;
};

}  // namespace b200ep
