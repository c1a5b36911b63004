#include "plan.h"

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <chrono>
#include <set>
#include <sstream>
#include <tuple>
#include <unordered_map>

#include "../common.cuh"
#include "../kernels/elementwise.h"
#include "../kernels/kernels.h"
#include "../kernels/mnb_mma.h"
#include "tp.h"

namespace b200ep {

DeviceErrorSlot* device_error_slot();

DevMem::~DevMem() {
  if (p) cudaFree(p);
}

int DevMem::alloc(size_t n) {
  if (cudaMalloc(&p, std::max<size_t>(n, 16)) != cudaSuccess) {
    cudaGetLastError();
    p = nullptr;
    return set_error(B200EP_ENOMEM, "device allocation of " + std::to_string(n) + " bytes failed");
  }
  bytes = n;
  return B200EP_OK;
}

struct Plan::Program {
  std::vector<Slot> slots;
  std::vector<std::unique_ptr<DevMem>> mems;
  std::map<std::string, cudaGraphExec_t> graphs;
  int path = 2;  // 0 decode, 1 prefill, 2 general (for the session summary)
  // integer glue evaluated on the host (no launch) and the host values that device steps read:
  // packed into one buffer uploaded by one copy per call (upl_*), plus output slots copied singly
  std::vector<char> host_step;
  std::vector<int> host_steps;
  std::vector<std::pair<int, size_t>> uploads;  // slot, offset in the packed buffer
  std::vector<int> out_uploads;
  std::vector<uint8_t> upl_host;
  void* upl_dev = nullptr;
  // the real extent of every input's changing key axis, read by the kernels from dims_dev
  std::map<int, int> dims_idx;  // slot -> index
  std::vector<int64_t> dims_host;
  int64_t* dims_dev = nullptr;
  ~Program() {
    for (auto& kv : graphs)
      if (kv.second) cudaGraphExecDestroy(kv.second);
  }
};

Plan::~Plan() {
  if (!prof_ms_.empty()) {
    double tot = 0;
    for (auto& kv : prof_ms_) tot += kv.second.second;
    std::vector<std::pair<double, std::string>> order;
    for (auto& kv : prof_ms_) order.push_back({-kv.second.second, kv.first});
    std::sort(order.begin(), order.end());
    fprintf(stderr, "[b200ep profile] rank %d: %.3f ms over %lld runs\n", cfg_.tp ? cfg_.tp->rank : 0, tot,
            (long long)stats_.runs);
    for (auto& [neg, name] : order) {
      auto& v = prof_ms_[name];
      fprintf(stderr, "[b200ep profile]   %-48s n=%6lld total=%9.3f ms avg=%8.2f us %5.1f%%\n", name.c_str(),
              (long long)v.first, v.second, v.second * 1e3 / v.first, 100.0 * v.second / tot);
    }
  }
  for (auto e : prof_ev_) cudaEventDestroy(e);
  programs_.clear();
  if (stream_) cudaStreamDestroy(stream_);
  if (ev_in_) cudaEventDestroy(ev_in_);
  if (ev_out_) cudaEventDestroy(ev_out_);
}

namespace {

std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? "," : "") + std::to_string(s[i]);
  return r + "]";
}

int64_t numel_of(const std::vector<int64_t>& s) {
  int64_t n = 1;
  for (auto d : s) n *= d;
  return n;
}

MnbAr make_ar(const TpContext& tp) {
  MnbAr a;
  a.world = tp.world;
  a.rank = tp.rank;
  a.ctrs = static_cast<unsigned*>(tp.ar_ctrs);
  for (int k = 0; k < tp.world; ++k) a.mbox[k] = static_cast<char*>(tp.ar_peer[k]);
  a.slot_bytes = tp.ar_slot_bytes;
  a.region_bytes = (size_t)tp.world * tp.ar_slot_bytes;
  return a;
}

bool env_on(const char* name) {
  const char* v = getenv(name);
  return v && *v && strcmp(v, "0") != 0;
}

}  // namespace

int Plan::slot_of(const std::string& name) {
  auto it = slot_index_.find(name);
  if (it != slot_index_.end()) return it->second;
  Slot s;
  s.name = name;
  slots_.push_back(s);
  slot_index_[name] = (int)slots_.size() - 1;
  return (int)slots_.size() - 1;
}

// ---- lowering -------------------------------------------------------------------------------
int Plan::lower(const Graph& g, const std::vector<int>& nodes, std::string* err) {
  std::set<std::string> produced;
  for (int ni : nodes)
    for (auto& o : g.nodes[ni].outputs)
      if (!o.empty()) produced.insert(o);
  std::set<int> inset(nodes.begin(), nodes.end());

  auto value_slot = [&](const std::string& name) -> int {
    if (name.empty()) return -1;
    auto it = slot_index_.find(name);
    if (it != slot_index_.end()) return it->second;
    int id = slot_of(name);
    Slot& s = slots_[id];
    if (auto* init = g.initializer(name)) {
      s.kind = Slot::kConst;
      s.dtype = init->dtype;
      s.cshape = init->shape;
      pending_consts_[id] = g.initializers.at(name);
    } else if (!produced.count(name)) {
      s.kind = Slot::kInput;
      s.io = (int)in_names_.size();
      in_names_.push_back(name);
      if (auto* vi = g.value(name)) s.dtype = vi->dtype;
    } else if (auto* vi = g.value(name)) {
      s.dtype = vi->dtype;
    }
    return id;
  };

  for (int ni : nodes) {
    const Node& n = g.nodes[ni];
    NodeView view(g, n);
    const OpEntry* e = find_entry(n.domain, n.op_type, g.opset(n.domain));
    if (!e) {
      *err = "no handler for " + n.op_type;
      return B200EP_EUNSUPPORTED;
    }
    Step st{};
    st.name = n.name.empty() ? n.op_type : n.name;
    for (auto& in : n.inputs) st.in.push_back(value_slot(in));
    for (auto& o : n.outputs) st.out.push_back(o.empty() ? -1 : value_slot(o));
    switch (e->kind) {
      case OpKind::kMatMulNBits: {
        st.kind = StepKind::kMnb;
        st.K = n.int_attr("K", 0);
        st.N = n.int_attr("N", 0);
        st.bits = (int)n.int_attr("bits", 4);
        st.block = (int)n.int_attr("block_size", 32);
        st.wB = st.in[1];
        st.wS = st.in[2];
        st.wZ = st.in.size() > 3 ? st.in[3] : -1;
        st.in.resize(1);
        st.out.resize(1);
        const int64_t nblocks = (st.K + st.block - 1) / st.block;
        const Initializer* B = g.initializer(n.inputs[1]);
        const Initializer* S = g.initializer(n.inputs[2]);
        if (!B || (int64_t)B->bytes.size() != st.N * nblocks * st.block * st.bits / 8) {
          *err = "MatMulNBits " + st.name + ": B has " + std::to_string(B ? B->bytes.size() : 0) +
                 " bytes, expected N*nblocks*block*bits/8";
          return B200EP_EINVAL;
        }
        if (!S || S->numel() != st.N * nblocks) {
          *err = "MatMulNBits " + st.name + ": scale count does not match N * nblocks";
          return B200EP_EINVAL;
        }
        if (st.wZ >= 0) {
          const Initializer* Z = g.initializer(n.inputs[3]);
          const int64_t zcols = st.bits == 4 ? (nblocks + 1) / 2 : nblocks;
          if (!Z || (int64_t)Z->bytes.size() != st.N * zcols) {
            *err = "MatMulNBits " + st.name + ": zero_points size does not match N * ceil(nblocks*bits/8)";
            return B200EP_EINVAL;
          }
        }
        break;
      }
      case OpKind::kGroupQueryAttention: {
        st.kind = StepKind::kGqa;
        st.num_heads = (int)n.int_attr("num_heads", 0);
        st.kv_heads = (int)n.int_attr("kv_num_heads", 0);
        st.packed = !n.input_present(1) && !n.input_present(2);
        const ValueInfo* q = view.input_info(0);
        st.head_size = (int)(st.packed ? q->shape[2] / (st.num_heads + 2 * st.kv_heads) : q->shape[2] / st.num_heads);
        st.do_rotary = (int)(n.int_attr("do_rotary", 1) != 0 && n.input_present(7));
        st.interleaved = (int)n.int_attr("rotary_interleaved", 0);
        st.local_window = (int)n.int_attr("local_window_size", -1);
        st.sliding = n.int_attr("sliding_window_cache", 0) != 0;
        st.scale = n.float_attr("scale", 0.f);
        st.qk_eps = n.float_attr("qk_norm_epsilon", 1e-6f);
        st.in.resize(16, -1);
        st.out.resize(3, -1);
        if (st.out[1] < 0 || st.out[2] < 0) {
          *err = "GroupQueryAttention " + st.name + ": present_key/present_value outputs are required";
          return B200EP_EUNSUPPORTED;
        }
        break;
      }
      case OpKind::kPagedAttention: {
        // inputs: q, k, v, key_cache, value_cache, cumulative lengths, past lengths, block table,
        // cos, sin; outputs: attention, key_cache / value_cache (the inputs updated in place)
        st.kind = StepKind::kPaged;
        st.num_heads = (int)n.int_attr("num_heads", 0);
        st.kv_heads = (int)n.int_attr("kv_num_heads", 0);
        st.head_size = (int)(view.input_info(0)->shape[1] / st.num_heads);
        st.do_rotary = (int)(n.int_attr("do_rotary", 0) != 0);
        st.interleaved = (int)n.int_attr("rotary_interleaved", 0);
        st.scale = n.float_attr("scale", 0.f);
        st.in.resize(10, -1);
        st.out.resize(3, -1);
        break;
      }
      case OpKind::kRmsNorm:
      case OpKind::kSimplifiedLayerNorm:
        st.kind = StepKind::kRms;
        st.eps = n.float_attr("epsilon", e->kind == OpKind::kRmsNorm ? 1e-6f : 1e-5f);
        st.out.resize(1);
        break;
      case OpKind::kSkipSimplifiedLayerNorm: {
        st.kind = StepKind::kRms;
        st.skip = true;
        st.eps = n.float_attr("epsilon", 1e-6f);
        // outputs: [0] normalised, [last] residual sum (norm.rs:241-245); mean/inv-std are never produced
        int residual = -1;
        if (n.outputs.size() >= 2) residual = st.out.back();
        for (size_t i = 1; i + 1 < n.outputs.size() && i < 3; ++i)
          if (!n.outputs[i].empty()) {
            const std::string& nm = n.outputs[i];
            bool used = g.is_graph_output(nm);
            for (auto& other : g.nodes)
              for (auto& in : other.inputs) used |= in == nm;
            if (used) {
              *err = "SkipSimplifiedLayerNormalization " + st.name + ": mean/inv_std_var outputs are consumed but not produced";
              return B200EP_EUNSUPPORTED;
            }
          }
        st.out = {st.out[0], residual};
        break;
      }
      case OpKind::kGatherBlockQuantized: {
        st.kind = StepKind::kGbq;
        st.block = (int)n.int_attr("block_size", 128);
        st.wB = st.in[0];
        st.wS = st.in[2];
        st.wZ = st.in.size() > 3 ? st.in[3] : -1;
        const Initializer* D = g.initializer(n.inputs[0]);
        st.gbq_rows = D->shape[0];
        st.gbq_dim = D->shape[1] * 2;
        st.in = {st.in[1]};
        st.out.resize(1);
        break;
      }
      case OpKind::kAdd:
      case OpKind::kSub:
      case OpKind::kMul:
        st.kind = StepKind::kBinary;
        st.bop = e->kind == OpKind::kAdd ? kOpAdd : e->kind == OpKind::kSub ? kOpSub : kOpMul;
        break;
      case OpKind::kSigmoid:
        st.kind = StepKind::kSigmoid;
        break;
      case OpKind::kCast:
        st.kind = StepKind::kCast;
        st.to = (int)n.int_attr("to", 0);
        break;
      case OpKind::kShape:
        st.kind = StepKind::kShape;
        st.shp_start = n.int_attr("start", 0);
        st.shp_end = n.int_attr("end", INT64_MAX);
        break;
      case OpKind::kGather: {
        st.kind = StepKind::kGatherIdx;
        const Initializer* idx = g.initializer(n.inputs[1]);
        st.ivals = const_ints(idx);
        st.idx_rank = (int)idx->shape.size();
        st.in.resize(1);
        break;
      }
      case OpKind::kReduceSum:
        st.kind = StepKind::kReduceSum;
        st.keepdims = n.int_attr("keepdims", 1) != 0;
        st.in.resize(1);
        break;
      case OpKind::kUnsqueeze:
      case OpKind::kSqueeze:
      case OpKind::kReshape:
        st.kind = StepKind::kCopy;
        st.layout = e->kind == OpKind::kUnsqueeze ? 1 : e->kind == OpKind::kSqueeze ? 2 : 3;
        st.ivals = n.input_present(1) ? const_ints(g.initializer(n.inputs[1])) : n.ints_attr("axes");
        st.in.resize(1);
        break;
    }
    steps_.push_back(std::move(st));
  }

  // boundary outputs: produced here and used outside the partition (or graph outputs)
  std::set<std::string> outside_uses;
  for (int ni = 0; ni < (int)g.nodes.size(); ++ni) {
    if (inset.count(ni)) continue;
    for (auto& in : g.nodes[ni].inputs) outside_uses.insert(in);
  }
  for (int ni : nodes)
    for (auto& o : g.nodes[ni].outputs) {
      if (o.empty()) continue;
      if (g.is_graph_output(o) || outside_uses.count(o)) {
        int id = slot_index_.at(o);
        Slot& s = slots_[id];
        s.kind = Slot::kOutput;
        s.io = (int)out_names_.size();
        out_names_.push_back(o);
        const ValueInfo* vi = g.value(o);
        out_dtypes_.push_back(vi ? vi->dtype : s.dtype);
        if (vi) s.dtype = vi->dtype;
      }
    }
  // dtypes of intermediates without value infos: inherit from the step's first float input
  for (auto& st : steps_)
    for (int o : st.out)
      if (o >= 0 && slots_[o].dtype == 0) {
        if (st.kind == StepKind::kCast) slots_[o].dtype = st.to;
        else if (st.kind == StepKind::kShape) slots_[o].dtype = kI64;
        else if (st.kind == StepKind::kGbq) slots_[o].dtype = slots_[st.wS].dtype;
        else if (!st.in.empty() && st.in[0] >= 0) slots_[o].dtype = slots_[st.in[0]].dtype;
      }
  return B200EP_OK;
}

// ---- fusion passes --------------------------------------------------------------------------
namespace {

struct Uses {
  std::vector<int> producer;            // slot -> step
  std::vector<std::vector<int>> users;  // slot -> steps
};

Uses uses_of(const std::vector<Step>& steps, size_t nslots) {
  Uses u;
  u.producer.assign(nslots, -1);
  u.users.assign(nslots, {});
  for (int i = 0; i < (int)steps.size(); ++i) {
    for (int o : steps[i].out)
      if (o >= 0) u.producer[o] = i;
    for (int s : steps[i].in)
      if (s >= 0) u.users[s].push_back(i);
  }
  return u;
}

// concatenate per-row weight arrays (rows along N) of several MatMulNBits initializers
std::shared_ptr<Initializer> concat_rows(const std::vector<std::shared_ptr<Initializer>>& parts,
                                         const std::string& name) {
  auto out = std::make_shared<Initializer>();
  out->name = name;
  out->dtype = parts[0]->dtype;
  int64_t rows = 0;
  size_t bytes = 0;
  for (auto& p : parts) {
    rows += p->shape.empty() ? 0 : p->shape[0];
    bytes += p->bytes.size();
  }
  out->shape = parts[0]->shape;
  if (!out->shape.empty()) out->shape[0] = rows;
  out->bytes.reserve(bytes);
  for (auto& p : parts) out->bytes.insert(out->bytes.end(), p->bytes.begin(), p->bytes.end());
  return out;
}

bool same_gemv_family(const Step& a, const Step& b) {
  return a.kind == StepKind::kMnb && b.kind == StepKind::kMnb && a.in[0] == b.in[0] && a.K == b.K &&
         a.bits == b.bits && a.block == b.block && (a.wZ >= 0) == (b.wZ >= 0);
}

}  // namespace

void Plan::fuse_qkv() {
  for (bool changed = true; changed;) {
    changed = false;
    Uses u = uses_of(steps_, slots_.size());
    for (int gi = 0; gi < (int)steps_.size() && !changed; ++gi) {
      Step& g = steps_[gi];
      if (g.kind != StepKind::kGqa || g.packed) continue;
      const int q = g.in[0], k = g.in[1], v = g.in[2];
      if (q < 0 || k < 0 || v < 0) continue;
      const int pq = u.producer[q], pk = u.producer[k], pv = u.producer[v];
      if (pq < 0 || pk < 0 || pv < 0 || pq == pk || pk == pv || pq == pv) continue;
      const Step &sq = steps_[pq], &sk = steps_[pk], &sv = steps_[pv];
      if (!same_gemv_family(sq, sk) || !same_gemv_family(sq, sv)) continue;
      bool private_outs = true;
      for (int s : {q, k, v}) private_outs &= slots_[s].kind == Slot::kTemp && u.users[s].size() == 1;
      if (!private_outs) continue;
      if (!pending_consts_.count(sq.wB) || !pending_consts_.count(sk.wB) || !pending_consts_.count(sv.wB)) continue;
      Step m = sq;
      m.name = sq.name + "+" + sk.name + "+" + sv.name;
      m.N = sq.N + sk.N + sv.N;
      auto cat = [&](int a, int b, int c, const std::string& nm) {
        int id = slot_of(nm);
        slots_[id].kind = Slot::kConst;
        auto init = concat_rows({pending_consts_[a], pending_consts_[b], pending_consts_[c]}, nm);
        slots_[id].dtype = init->dtype;
        slots_[id].cshape = init->shape;
        pending_consts_[id] = init;
        return id;
      };
      m.wB = cat(sq.wB, sk.wB, sv.wB, m.name + "#B");
      m.wS = cat(sq.wS, sk.wS, sv.wS, m.name + "#scales");
      if (sq.wZ >= 0) m.wZ = cat(sq.wZ, sk.wZ, sv.wZ, m.name + "#zp");
      const int qkv = slot_of(m.name + "#qkv");
      slots_[qkv].dtype = slots_[q].dtype;
      m.out = {qkv};
      g.in[0] = qkv;
      g.in[1] = g.in[2] = -1;
      g.packed = true;
      const int first = std::min({pq, pk, pv});
      std::vector<int> drop = {pq, pk, pv};
      std::sort(drop.rbegin(), drop.rend());
      for (int d : drop) steps_.erase(steps_.begin() + d);
      steps_.insert(steps_.begin() + first, m);
      ++stats_.fused_qkv;
      changed = true;
    }
  }
}

void Plan::fuse_swiglu() {
  for (bool changed = true; changed;) {
    changed = false;
    Uses u = uses_of(steps_, slots_.size());
    for (int i3 = 0; i3 < (int)steps_.size() && !changed; ++i3) {
      const Step& m3 = steps_[i3];
      if (m3.kind != StepKind::kBinary || m3.bop != kOpMul || m3.in.size() != 2) continue;
      for (int order = 0; order < 2 && !changed; ++order) {
        const int silu = m3.in[order], up = m3.in[1 - order];
        const int i2 = u.producer[silu];
        if (i2 < 0 || steps_[i2].kind != StepKind::kBinary || steps_[i2].bop != kOpMul) continue;
        const Step& m2 = steps_[i2];
        int gate = -1, sig = -1;
        for (int o2 = 0; o2 < 2; ++o2) {
          const int a = m2.in[o2], b = m2.in[1 - o2];
          const int is = u.producer[b];
          if (is >= 0 && steps_[is].kind == StepKind::kSigmoid && steps_[is].in[0] == a) {
            gate = a;
            sig = b;
          }
        }
        if (gate < 0) continue;
        const int isg = u.producer[sig];
        const int pg = u.producer[gate], pu = u.producer[up];
        if (pg < 0 || pu < 0 || pg == pu) continue;
        const Step &sg = steps_[pg], &su = steps_[pu];
        if (!same_gemv_family(sg, su) || sg.N != su.N) continue;
        bool private_vals = true;
        for (int s : {gate, sig, silu, up}) private_vals &= slots_[s].kind == Slot::kTemp;
        private_vals &= u.users[gate].size() == 2 && u.users[sig].size() == 1 && u.users[silu].size() == 1 &&
                        u.users[up].size() == 1;
        if (!private_vals) continue;
        if (slots_[m3.out[0]].dtype != slots_[gate].dtype) continue;
        Step m = sg;
        m.name = sg.name + "+" + su.name;
        m.N = sg.N + su.N;
        auto cat = [&](int a, int b, const std::string& nm) {
          int id = slot_of(nm);
          slots_[id].kind = Slot::kConst;
          auto init = concat_rows({pending_consts_[a], pending_consts_[b]}, nm);
          slots_[id].dtype = init->dtype;
          slots_[id].cshape = init->shape;
          pending_consts_[id] = init;
          return id;
        };
        m.wB = cat(sg.wB, su.wB, m.name + "#B");
        m.wS = cat(sg.wS, su.wS, m.name + "#scales");
        if (sg.wZ >= 0) m.wZ = cat(sg.wZ, su.wZ, m.name + "#zp");
        const int gu = slot_of(m.name + "#gate_up");
        slots_[gu].dtype = slots_[gate].dtype;
        m.out = {gu};
        Step act{};
        act.kind = StepKind::kSiluMul;
        act.name = m.name + "#swiglu";
        act.in = {gu};
        act.out = {m3.out[0]};
        act.N = sg.N;
        std::vector<int> drop = {pg, pu, isg, i2, i3};
        const int first = std::min(pg, pu);
        std::sort(drop.rbegin(), drop.rend());
        for (int d : drop) steps_.erase(steps_.begin() + d);
        // act goes where m3 was (after removals, positions before i3 shift by the drops before it)
        int pos_act = i3;
        for (int d : drop)
          if (d < i3) --pos_act;
        steps_.insert(steps_.begin() + pos_act, act);
        int pos_m = first;
        steps_.insert(steps_.begin() + std::min<int>(pos_m, pos_act), m);
        ++stats_.fused_swiglu;
        changed = true;
      }
    }
  }
}

// The fused gate/up GEMV followed by SiLU(gate) * up (after tensor-parallel slicing, before the
// upload): reorder the weight rows so that every 16-row tile holds 8 gate rows and the 8 matching up
// rows, and let the GEMV's tile merge write h = SiLU(gate) * up itself.  The separate SiLU step
// (or the down projection's SiLU prologue, which re-read the 2F-wide gate/up output in every CTA)
// goes away.  Only for weights the tensor-core GEMV takes (the other paths still work through the
// workspace and the interleaved SiLU kernel).
void Plan::fuse_swiglu_epilogue() {
  Uses u = uses_of(steps_, slots_.size());
  for (int ai = 0; ai < (int)steps_.size(); ++ai) {
    const Step a = steps_[ai];
    if (a.kind != StepKind::kSiluMul) continue;
    const int gu = a.in[0], pi = u.producer[gu];
    if (pi < 0 || u.users[gu].size() != 1 || slots_[gu].kind != Slot::kTemp) continue;
    Step& m = steps_[pi];
    const int64_t F = a.N;
    if (m.kind != StepKind::kMnb || m.N != 2 * F || F % 8 || m.in.empty() || m.in[0] < 0) continue;
    if (!mnb_mma_supported(slots_[m.in[0]].dtype, m.bits, m.block, m.K)) continue;
    bool have = true;
    for (int w : {m.wB, m.wS, m.wZ})
      if (w >= 0) have &= pending_consts_.count(w) && (int64_t)pending_consts_[w]->bytes.size() % m.N == 0;
    if (!have) continue;
    // row 16 i + r <- gate row 8 i + r, row 16 i + 8 + r <- up row 8 i + r (r < 8); up rows are F .. 2F
    auto interleave = [&](int id, const std::string& nm) {
      const Initializer& in = *pending_consts_[id];
      const size_t rb = in.bytes.size() / (size_t)m.N;
      auto out = std::make_shared<Initializer>();
      out->name = nm;
      out->dtype = in.dtype;
      out->shape = in.shape;
      out->bytes.resize(in.bytes.size());
      for (int64_t i = 0; i < F / 8; ++i)
        for (int r = 0; r < 16; ++r) {
          const int64_t src = r < 8 ? 8 * i + r : F + 8 * i + (r - 8);
          memcpy(out->bytes.data() + (size_t)(16 * i + r) * rb, in.bytes.data() + (size_t)src * rb, rb);
        }
      const int nid = slot_of(nm);
      slots_[nid].kind = Slot::kConst;
      slots_[nid].dtype = out->dtype;
      slots_[nid].cshape = out->shape;
      pending_consts_[nid] = out;
      return nid;
    };
    m.wB = interleave(m.wB, m.name + "#B#swiglu");
    m.wS = interleave(m.wS, m.name + "#scales#swiglu");
    if (m.wZ >= 0) m.wZ = interleave(m.wZ, m.name + "#zp#swiglu");
    m.swiglu = true;
    ++stats_.swiglu_epilogue;
    m.out = {a.out[0]};
    const int ws = slot_of(m.name + "#gate_up_interleaved");
    slots_[ws].dtype = slots_[gu].dtype;
    m.ws_slot = ws;
    steps_.erase(steps_.begin() + ai);
    u = uses_of(steps_, slots_.size());
    --ai;
  }
}

int Plan::upload_constants(const Graph& g, std::string* err) {
  // fp16 / bf16 int4 MatMulNBits: upload the ORT-layout weight once, repack it on the device into
  // the tensor-core operand order, keep only the packed form
  for (auto& st : steps_) {
    if (st.kind != StepKind::kMnb || st.in.empty() || st.in[0] < 0) continue;
    const int adt = slots_[st.in[0]].dtype;
    if (env_on("ONNXRUNTIME_EP_B200_NO_PREPACK") || !mnb_mma_supported(adt, st.bits, st.block, st.K)) continue;
    auto host = [&](int id) { return pending_consts_.count(id) ? pending_consts_[id] : nullptr; };
    auto B = host(st.wB), S = host(st.wS), Z = st.wZ >= 0 ? host(st.wZ) : nullptr;
    if (!B || !S || (st.wZ >= 0 && !Z)) continue;
    MnbPacked pk = mnb_packed_geometry(st.N, st.K, st.block);
    DevMem tb, ts, tz;
    st.pk_w = std::make_shared<DevMem>();
    int rc = 0;
    rc |= tb.alloc(B->bytes.size());
    rc |= ts.alloc(S->bytes.size());
    if (Z) rc |= tz.alloc(Z->bytes.size());
    rc |= st.pk_w->alloc(pk.bytes);
    if (rc) {
      *err = "weight upload: out of device memory";
      return B200EP_ENOMEM;
    }
    cudaError_t e = cudaMemcpy(tb.p, B->bytes.data(), B->bytes.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(ts.p, S->bytes.data(), S->bytes.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && Z) e = cudaMemcpy(tz.p, Z->bytes.data(), Z->bytes.size(), cudaMemcpyHostToDevice);
    pk.w = st.pk_w->p;
    if (e == cudaSuccess)
      e = launch_mnb_prepack(static_cast<const uint8_t*>(tb.p), ts.p, Z ? static_cast<const uint8_t*>(tz.p) : nullptr,
                             adt, pk, nullptr);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      *err = std::string("weight prepack failed: ") + cudaGetErrorString(e);
      return B200EP_ECUDA;
    }
    st.prepacked = true;
    stats_.weight_bytes += (int64_t)pk.bytes;
  }
  std::set<int> used;
  for (auto& st : steps_) {
    if (st.kind == StepKind::kMnb && st.prepacked) continue;
    for (int s : st.in)
      if (s >= 0 && slots_[s].kind == Slot::kConst) used.insert(s);
    for (int s : {st.wB, st.wS, st.wZ})
      if (s >= 0) used.insert(s);
  }
  for (int id : used) {
    auto it = pending_consts_.find(id);
    if (it == pending_consts_.end()) {
      *err = "constant " + slots_[id].name + " has no data";
      return B200EP_EINTERNAL;
    }
    auto mem = std::make_shared<DevMem>();
    int rc = mem->alloc(it->second->bytes.size());
    if (rc) {
      *err = "weight upload: out of device memory";
      return rc;
    }
    if (!it->second->bytes.empty() &&
        cudaMemcpy(mem->p, it->second->bytes.data(), it->second->bytes.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
      *err = "weight upload failed";
      return B200EP_ECUDA;
    }
    slots_[id].cmem = mem;
    slots_[id].ptr = mem->p;
    slots_[id].shape = slots_[id].cshape;
    if (it->second->bytes.size() <= 64) slots_[id].host_copy = it->second->bytes;
    stats_.weight_bytes += (int64_t)it->second->bytes.size();
  }
  pending_consts_.clear();
  return B200EP_OK;
}

std::string SessionSummary::json() const {
  std::lock_guard<std::mutex> lk(mu);
  std::ostringstream o;
  o << "{\"getcap_calls\":" << getcap_calls << ",\"total_nodes\":" << total_nodes
    << ",\"claimed_nodes\":" << claimed_nodes << ",\"partitions\":" << partitions << ",\"rejected\":{";
  bool first = true;
  for (auto& [op, v] : rejected) {
    o << (first ? "" : ",") << "\"" << op << "\":{\"nodes\":" << v.first << ",\"reason\":\"";
    for (char ch : v.second) o << (ch == '"' || ch == '\\' ? '\'' : ch);
    o << "\"}";
    first = false;
  }
  o << "},\"compiles\":" << compiles << ",\"compile_ms\":" << compile_ms << ",\"weight_bytes\":" << weight_bytes
    << ",\"path_decode\":" << path_decode << ",\"path_prefill\":" << path_prefill
    << ",\"path_general\":" << path_general << ",\"graph_replays\":" << graph_replays
    << ",\"graph_captures\":" << graph_captures << ",\"eager_runs\":" << eager_runs
    << ",\"key_hits\":" << key_hits << ",\"key_misses\":" << key_misses << ",\"h2d_bytes\":" << h2d_bytes
    << ",\"d2h_bytes\":" << d2h_bytes << ",\"run_ms\":" << run_ms << "}";
  return o.str();
}

std::string SessionSummary::text() const {
  std::lock_guard<std::mutex> lk(mu);
  std::ostringstream o;
  const double pct = total_nodes ? 100.0 * (double)claimed_nodes / (double)total_nodes : 0.0;
  o.setf(std::ios::fixed);
  o.precision(1);
  o << "===== B200 EP session summary =====\n"
    << "  claim:   " << claimed_nodes << "/" << total_nodes << " nodes claimed (" << pct << "%) across "
    << partitions << " partition(s), " << getcap_calls << " GetCapability call(s)\n";
  if (!rejected.empty()) {
    o << "           unclaimed (-> CPU):\n";
    for (auto& [op, v] : rejected) o << "             - " << op << " x" << v.first << ": " << v.second << "\n";
  }
  o << "  compile: " << compiles << " partition(s), " << compile_ms << " ms, "
    << (double)weight_bytes / (1024.0 * 1024.0) << " MiB of weights in HBM\n"
    << "  compute: decode=" << path_decode << " prefill=" << path_prefill << " general=" << path_general
    << "  (graph replay " << graph_replays << ", capture " << graph_captures << ", eager " << eager_runs
    << "; shape keys " << key_hits << " HIT / " << key_misses << " MISS)\n"
    << "  memory:  host inputs staged " << (double)h2d_bytes / (1024.0 * 1024.0) << " MiB H2D, host outputs "
    << (double)d2h_bytes / (1024.0 * 1024.0) << " MiB D2H\n"
    << "  timing:  compile=" << compile_ms << " ms, run (host)=" << run_ms << " ms\n"
    << "===================================";
  return o.str();
}

std::unique_ptr<Plan> Plan::compile(const Graph& g, const std::vector<int>& nodes, const EpConfig& cfg,
                                    std::string* err) {
  const auto t0 = std::chrono::steady_clock::now();
  std::unique_ptr<Plan> p = compile_impl(g, nodes, cfg, err);
  if (p && cfg.summary && !cfg.host_only) {
    std::lock_guard<std::mutex> lk(cfg.summary->mu);
    ++cfg.summary->compiles;
    cfg.summary->weight_bytes += p->stats_.weight_bytes;
    cfg.summary->compile_ms +=
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  }
  return p;
}

std::unique_ptr<Plan> Plan::compile_impl(const Graph& g, const std::vector<int>& nodes, const EpConfig& cfg,
                                         std::string* err) {
  std::unique_ptr<Plan> p(new Plan());
  p->cfg_ = cfg;
  p->prof_ = env_on("ONNXRUNTIME_EP_B200_PROFILE");
  p->stats_.nodes = (int)nodes.size();
  if (p->lower(g, nodes, err)) return nullptr;
  if (cfg.fuse && !env_on("ONNXRUNTIME_EP_B200_NO_FUSION")) {
    p->fuse_qkv();
    p->fuse_swiglu();
  }
  if (cfg.tp && p->shard_for_tp(err)) return nullptr;
  if (cfg.host_only) return p;
  if (cfg.fuse && !env_on("ONNXRUNTIME_EP_B200_NO_FUSION") && !env_on("ONNXRUNTIME_EP_B200_NO_SWIGLU_EPILOGUE"))
    p->fuse_swiglu_epilogue();
  if (p->upload_constants(g, err)) return nullptr;
  if (cfg.fuse) {
    p->fuse_prologues();
    p->fuse_peer_allreduce();
  }
  p->compute_free_rules();
  p->stats_.steps = (int)p->steps_.size();
  if (cfg.verbose) fprintf(stderr, "[b200ep] compiled partition: %s\n", p->describe().c_str());
  return p;
}

void Plan::fuse_prologues() {
  for (bool changed = true; changed;) {
    changed = false;
    Uses u = uses_of(steps_, slots_.size());
    for (int im = 0; im < (int)steps_.size() && !changed; ++im) {
      Step& m = steps_[im];
      if (m.kind != StepKind::kMnb || !m.prepacked || m.pro) continue;
      const int a = m.in[0];
      const int ip = u.producer[a];
      if (ip < 0 || ip >= im || slots_[a].kind != Slot::kTemp || u.users[a].size() != 1) continue;
      const Step& p = steps_[ip];
      if (p.kind == StepKind::kRms) {
        // the residual output (skip form) is now written by the GEMV: its readers must follow it
        const int res = p.skip && p.out.size() > 1 ? p.out[1] : -1;
        bool ok = true;
        if (res >= 0)
          for (int r : u.users[res]) ok &= r > im;
        // nothing between the norm and the GEMV may overwrite the norm's inputs
        for (int k = ip + 1; k < im && ok; ++k)
          for (int o : steps_[k].out)
            for (int i : p.in) ok &= o != i;
        if (!ok) continue;
        m.pro = p.skip ? kProSkipRms : kProRms;
        m.pro_x = p.in[0];
        m.pro_skip = p.skip ? p.in[1] : -1;
        m.pro_gamma = p.in[p.skip ? 2 : 1];
        m.pro_res = res;
        m.pro_eps = p.eps;
        ++stats_.fused_norm;
      } else if (p.kind == StepKind::kSiluMul && p.N == m.K) {
        bool ok = true;
        for (int k = ip + 1; k < im && ok; ++k)
          for (int o : steps_[k].out) ok &= o != p.in[0];
        if (!ok) continue;
        m.pro = kProSiluMul;
        m.pro_x = p.in[0];
        m.pro_n = p.N;
        ++stats_.fused_act;
      } else {
        continue;
      }
      m.name = p.name + ">" + m.name;
      steps_.erase(steps_.begin() + ip);
      changed = true;
    }
  }
}

bool Plan::ar_fused(int64_t M, int64_t hidden, int cons_block) const {
  return cfg_.tp && cfg_.tp->ar_ok && M >= 1 && M <= 16 && hidden % 8 == 0 &&
         (size_t)(M * hidden * 2) <= cfg_.tp->ar_slot_bytes &&
         mnb_prologue_fits(M, hidden, cons_block);
}

void Plan::fuse_peer_allreduce() {
  if (!cfg_.tp || !cfg_.tp->ar_ok) return;
  Uses u = uses_of(steps_, slots_.size());
  // readers of a slot, counting the inputs folded into GEMV prologues
  auto readers = [&](int slot) {
    std::vector<int> r = u.users[slot];
    for (int i = 0; i < (int)steps_.size(); ++i)
      for (int x : {steps_[i].pro_x, steps_[i].pro_skip, steps_[i].pro_gamma})
        if (x == slot) r.push_back(i);
    return r;
  };
  for (int ai = 0; ai < (int)steps_.size(); ++ai) {
    Step& a = steps_[ai];
    if (a.kind != StepKind::kAllReduce) continue;
    const int ip = u.producer[a.in[0]];
    if (ip < 0 || steps_[ip].kind != StepKind::kMnb || !steps_[ip].prepacked || steps_[ip].ar_out) continue;
    const std::vector<int> rd = readers(a.out[0]);
    if (rd.size() != 1 || slots_[a.out[0]].kind != Slot::kTemp) continue;
    const int im = rd[0];
    Step& m = steps_[im];
    if (m.kind != StepKind::kMnb || !m.prepacked || m.pro != kProSkipRms || m.pro_x != a.out[0] || im < ai) continue;
    // the consumer pairs with the latest producer: no other mailbox producer in between
    bool clear = true;
    for (int k = ip + 1; k < im; ++k) clear &= !steps_[k].ar_out;
    if (!clear) continue;
    Step& p = steps_[ip];
    p.ar_out = true;
    p.ar_block = m.block;
    a.ar_skip = true;
    a.ar_block = m.block;
    m.pro_ar = true;
    ++stats_.peer_allreduce;
  }
}

namespace {

// Row / block slicing of MatMulNBits initializers (ORT layout: B [N, nblocks, block*bits/8],
// scales [N * nblocks] or [N, nblocks], zero points [N, ceil(nblocks/2)] packed int4 or [N, nblocks]).
std::shared_ptr<Initializer> slice_rows(const Initializer& in, int64_t n_total,
                                        const std::vector<std::pair<int64_t, int64_t>>& ranges,
                                        const std::string& name) {
  auto out = std::make_shared<Initializer>();
  out->name = name;
  out->dtype = in.dtype;
  const size_t row_bytes = in.bytes.size() / (size_t)n_total;
  int64_t rows = 0;
  for (auto [a, b] : ranges) {
    out->bytes.insert(out->bytes.end(), in.bytes.begin() + a * row_bytes, in.bytes.begin() + b * row_bytes);
    rows += b - a;
  }
  out->shape = in.shape;
  if (in.shape.size() >= 2 && in.shape[0] == n_total)
    out->shape[0] = rows;
  else
    out->shape = {in.numel() / n_total * rows};
  return out;
}

// blocks [b0, b1) of every row; elem_bits = bits per block entry (B: block*bits, scales: 8*esz,
// packed int4 zero points: 4)
std::shared_ptr<Initializer> slice_blocks(const Initializer& in, int64_t n, int64_t nblocks, int64_t b0, int64_t b1,
                                          int elem_bits, const std::string& name) {
  auto out = std::make_shared<Initializer>();
  out->name = name;
  out->dtype = in.dtype;
  const int64_t nb = b1 - b0;
  const size_t in_row = in.bytes.size() / (size_t)n;
  if (elem_bits % 8 == 0) {
    const size_t eb = elem_bits / 8;
    for (int64_t r = 0; r < n; ++r) {
      const uint8_t* src = in.bytes.data() + r * in_row + b0 * eb;
      out->bytes.insert(out->bytes.end(), src, src + nb * eb);
    }
  } else {  // packed nibbles, low nibble = even block
    const size_t out_row = (size_t)(nb + 1) / 2;
    out->bytes.assign(out_row * n, 0);
    for (int64_t r = 0; r < n; ++r)
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t byte = in.bytes[r * in_row + (b0 + b) / 2];
        const uint8_t nib = ((b0 + b) & 1) ? (byte >> 4) : (byte & 0x0f);
        out->bytes[r * out_row + b / 2] |= (uint8_t)((b & 1) ? nib << 4 : nib);
      }
  }
  if (in.shape.size() == 3) out->shape = {n, nb, in.shape[2]};
  else if (in.shape.size() == 2) out->shape = {n, (int64_t)(out->bytes.size() / n)};
  else out->shape = {(int64_t)out->bytes.size() / std::max(1, dtype_size(in.dtype))};
  return out;
}

}  // namespace

namespace {
bool packed_inputs(const Step& g) { return g.packed; }
}  // namespace

int Plan::shard_for_tp(std::string* err) {
  if (!cfg_.tp || cfg_.tp->world == 1) return B200EP_OK;
  const int W = cfg_.tp->world, rk = cfg_.tp->rank;
  auto fail = [&](const std::string& m) {
    *err = "tensor parallel (" + std::to_string(W) + " ranks): " + m;
    return B200EP_EUNSUPPORTED;
  };
  for (const Step& s : steps_)
    if (s.kind == StepKind::kPaged) return fail(s.name + ": PagedAttention caches are not sharded");
  auto replace_const = [&](int id, std::shared_ptr<Initializer> init) {
    const int nid = slot_of(init->name);
    slots_[nid].kind = Slot::kConst;
    slots_[nid].dtype = init->dtype;
    slots_[nid].cshape = init->shape;
    pending_consts_[nid] = init;
    (void)id;
    return nid;
  };
  // column split: keep output rows `ranges` of step m
  auto split_cols = [&](Step& m, const std::vector<std::pair<int64_t, int64_t>>& ranges) -> int {
    for (int w : {m.wB, m.wS, m.wZ})
      if (w >= 0 && !pending_consts_.count(w)) return fail(m.name + ": weights not available for slicing");
    const std::string tag = "#tp" + std::to_string(rk) + "of" + std::to_string(W);
    m.wB = replace_const(m.wB, slice_rows(*pending_consts_[m.wB], m.N, ranges, m.name + "#B" + tag));
    m.wS = replace_const(m.wS, slice_rows(*pending_consts_[m.wS], m.N, ranges, m.name + "#scales" + tag));
    if (m.wZ >= 0) m.wZ = replace_const(m.wZ, slice_rows(*pending_consts_[m.wZ], m.N, ranges, m.name + "#zp" + tag));
    int64_t n = 0;
    for (auto [a, b] : ranges) n += b - a;
    m.N = n;
    return B200EP_OK;
  };
  // row split: keep input columns [k0, k1) of step m (block aligned)
  auto split_k = [&](Step& m, int64_t k0, int64_t k1) -> int {
    if (k0 % m.block || k1 % m.block || m.K % m.block) return fail(m.name + ": K shard not block aligned");
    for (int w : {m.wB, m.wS, m.wZ})
      if (w >= 0 && !pending_consts_.count(w)) return fail(m.name + ": weights not available for slicing");
    const int64_t nblocks = m.K / m.block, b0 = k0 / m.block, b1 = k1 / m.block;
    const std::string tag = "#tp" + std::to_string(rk) + "of" + std::to_string(W);
    m.wB = replace_const(m.wB, slice_blocks(*pending_consts_[m.wB], m.N, nblocks, b0, b1, m.block * m.bits,
                                            m.name + "#B" + tag));
    const Initializer& sc = *pending_consts_[m.wS];
    m.wS = replace_const(m.wS, slice_blocks(sc, m.N, nblocks, b0, b1, 8 * dtype_size(sc.dtype),
                                            m.name + "#scales" + tag));
    if (m.wZ >= 0)
      m.wZ = replace_const(m.wZ, slice_blocks(*pending_consts_[m.wZ], m.N, nblocks, b0, b1, m.bits == 4 ? 4 : 8,
                                              m.name + "#zp" + tag));
    m.K = k1 - k0;
    return B200EP_OK;
  };
  std::vector<int> row_parallel;  // steps whose partial sums need an all-reduce
  std::set<int> done;
  Uses u = uses_of(steps_, slots_.size());
  for (int gi = 0; gi < (int)steps_.size(); ++gi) {
    Step& g = steps_[gi];
    if (g.kind != StepKind::kGqa) continue;
    if (cfg_.tp_replicate_attention) {
      // attention runs in full on every rank: its projections are kept whole (not sharded, and
      // not taken by the vocabulary split below)
      Uses uu = uses_of(steps_, slots_.size());
      for (int j = 0; j < (packed_inputs(g) ? 1 : 3); ++j)
        if (uu.producer[g.in[j]] >= 0) done.insert(uu.producer[g.in[j]]);
      for (int c : uu.users[g.out[0]]) done.insert(c);
      continue;
    }
    const int H = g.num_heads, HK = g.kv_heads, D = g.head_size;
    if (H % W || HK % W) return fail("attention heads " + std::to_string(H) + "/" + std::to_string(HK) +
                                     " do not divide over the ranks");
    const int64_t hq = H / W, hk = HK / W;
    if (g.packed) {
      const int p = u.producer[g.in[0]];
      if (p < 0 || steps_[p].kind != StepKind::kMnb || steps_[p].N != (int64_t)(H + 2 * HK) * D)
        return fail(g.name + ": packed q/k/v does not come from one MatMulNBits");
      if (int rc = split_cols(steps_[p], {{rk * hq * D, (rk + 1) * hq * D},
                                          {(int64_t)H * D + rk * hk * D, (int64_t)H * D + (rk + 1) * hk * D},
                                          {(int64_t)(H + HK) * D + rk * hk * D, (int64_t)(H + HK) * D + (rk + 1) * hk * D}}))
        return rc;
      done.insert(p);
    } else {
      const int64_t per[3] = {hq, hk, hk};
      for (int j = 0; j < 3; ++j) {
        const int p = u.producer[g.in[j]];
        if (p < 0 || steps_[p].kind != StepKind::kMnb) return fail(g.name + ": q/k/v do not come from MatMulNBits");
        if (int rc = split_cols(steps_[p], {{rk * per[j] * D, (rk + 1) * per[j] * D}})) return rc;
        done.insert(p);
      }
    }
    g.num_heads = (int)hq;
    g.kv_heads = (int)hk;
    for (int c : u.users[g.out[0]]) {
      Step& o = steps_[c];
      if (o.kind != StepKind::kMnb || o.in[0] != g.out[0] || done.count(c)) return fail(g.name + ": output consumer");
      if (int rc = split_k(o, rk * hq * D, (rk + 1) * hq * D)) return rc;
      done.insert(c);
      row_parallel.push_back(c);
    }
  }
  for (int ai = 0; ai < (int)steps_.size(); ++ai) {
    Step& a = steps_[ai];
    if (a.kind != StepKind::kSiluMul) continue;
    const int64_t F = a.N;
    if (F % W) return fail("FFN width does not divide over the ranks");
    const int64_t f = F / W;
    const int p = u.producer[a.in[0]];
    if (p < 0 || steps_[p].kind != StepKind::kMnb || steps_[p].N != 2 * F) return fail(a.name + ": gate/up producer");
    if (int rc = split_cols(steps_[p], {{rk * f, (rk + 1) * f}, {F + rk * f, F + (rk + 1) * f}})) return rc;
    done.insert(p);
    a.N = f;
    for (int c : u.users[a.out[0]]) {
      Step& d = steps_[c];
      if (d.kind != StepKind::kMnb || d.in[0] != a.out[0] || done.count(c)) return fail(a.name + ": output consumer");
      if (int rc = split_k(d, rk * f, (rk + 1) * f)) return rc;
      done.insert(c);
      row_parallel.push_back(c);
    }
  }
  // vocabulary-split projection onto a partition output, then an all-gather of the logits
  std::vector<int> gathered;
  for (int li = 0; li < (int)steps_.size(); ++li) {
    Step& l = steps_[li];
    if (l.kind != StepKind::kMnb || done.count(li) || slots_[l.out[0]].kind != Slot::kOutput || l.N % W) continue;
    const int64_t n = l.N / W, full = l.N;
    if (int rc = split_cols(l, {{rk * n, (rk + 1) * n}})) return rc;
    l.shard_cols = full;  // remembered for the gather step
    done.insert(li);
    gathered.push_back(li);
  }
  // insert the collectives after their producers (back to front keeps the indices valid)
  std::vector<std::pair<int, Step>> ins;
  for (int c : row_parallel) {
    Step& m = steps_[c];
    const int out = m.out[0];
    const int part = slot_of(m.name + "#partial");
    slots_[part].dtype = slots_[out].dtype;
    m.out[0] = part;
    Step ar{};
    ar.kind = StepKind::kAllReduce;
    ar.name = m.name + "#allreduce";
    ar.in = {part};
    ar.out = {out};
    ins.push_back({c, ar});
  }
  for (int li : gathered) {
    Step& l = steps_[li];
    const int out = l.out[0];
    const int shard = slot_of(l.name + "#shard");
    const int stage = slot_of(l.name + "#gather");
    slots_[shard].dtype = slots_[stage].dtype = slots_[out].dtype;
    l.out[0] = shard;
    Step ag{};
    ag.kind = StepKind::kAllGather;
    ag.name = l.name + "#allgather";
    ag.in = {shard};
    ag.out = {out};
    ag.N = l.shard_cols;
    ag.shard_cols = l.N;
    ag.ws_slot = stage;
    l.shard_cols = 0;
    ins.push_back({li, ag});
  }
  std::sort(ins.begin(), ins.end(), [](auto& x, auto& y) { return x.first > y.first; });
  for (auto& [pos, st] : ins) steps_.insert(steps_.begin() + pos + 1, st);
  return B200EP_OK;
}

// ---- shape inference ------------------------------------------------------------------------
namespace {

const char* step_kind_name(StepKind k) {
  static const char* names[] = {"MatMulNBits", "GroupQueryAttention", "RmsNorm", "Binary", "Sigmoid", "SiluMul",
                                "Cast", "GatherBlockQuantized", "AllReduce", "AllGather", "PagedAttention",
                                "Shape", "Gather", "ReduceSum", "Copy"};
  return names[(int)k];
}

bool is_int_dtype(int dt) { return dt == kI32 || dt == kI64; }

// values of a little-endian int32 / int64 byte image
std::vector<int64_t> ints_of(const std::vector<uint8_t>& bytes, int dtype) {
  std::vector<int64_t> v;
  if (dtype == kI64) {
    v.resize(bytes.size() / 8);
    memcpy(v.data(), bytes.data(), v.size() * 8);
  } else if (dtype == kI32) {
    for (size_t i = 0; i + 4 <= bytes.size(); i += 4) {
      int32_t x;
      memcpy(&x, bytes.data() + i, 4);
      v.push_back(x);
    }
  }
  return v;
}

// host values of the integer constants and of host-resident integer scalars
void seed_host_values(std::vector<Slot>& S) {
  for (auto& s : S) {
    if ((s.kind == Slot::kConst || s.kind == Slot::kInput) && is_int_dtype(s.dtype) && !s.host_copy.empty()) {
      s.hval = ints_of(s.host_copy, s.dtype);
      s.hknown = (int64_t)s.hval.size() == numel_of(s.kind == Slot::kConst ? s.cshape : s.shape);
    } else if (s.kind != Slot::kConst) {
      s.hknown = false;
      s.hval.clear();
    }
  }
}

// integer a op b, ONNX wrap-around for int32
int64_t int_op(int op, int64_t a, int64_t b, int dtype) {
  const int64_t r = op == kOpAdd ? (int64_t)((uint64_t)a + (uint64_t)b)
                                 : op == kOpSub ? (int64_t)((uint64_t)a - (uint64_t)b) : (int64_t)((uint64_t)a * (uint64_t)b);
  return dtype == kI32 ? (int64_t)(int32_t)(uint32_t)(uint64_t)r : r;
}

}  // namespace

int Plan::infer_glue(const Step& st, std::vector<Slot>& S, std::string* err) const {
  auto fail = [&](const std::string& m) {
    *err = m;
    return B200EP_EINVAL;
  };
  Slot& y = S[st.out[0]];
  const Slot& x = S[st.in[0]];
  const auto& xs = x.rshape.empty() ? x.shape : x.rshape;  // a changing key axis: this call's extent
  switch (st.kind) {
    case StepKind::kShape: {
      // rust/src/ops/shape.rs:948-961, shape_interval :971-980
      const int64_t rank = (int64_t)xs.size();
      int64_t a = st.shp_start, b = st.shp_end == INT64_MAX ? rank : st.shp_end;
      a = std::clamp<int64_t>(a < 0 ? a + rank : a, 0, rank);
      b = std::clamp<int64_t>(b < 0 ? b + rank : b, 0, rank);
      y.shape = {std::max<int64_t>(b - a, 0)};
      y.hval.assign(xs.begin() + a, xs.begin() + std::max(a, b));
      y.hknown = true;
      return B200EP_OK;
    }
    case StepKind::kGatherIdx: {
      if (x.shape.size() != 1) return fail("Gather " + st.name + ": data must be 1-D");
      const int64_t n = x.shape[0];
      std::vector<int64_t> idx;
      for (int64_t i : st.ivals) {
        const int64_t j = i < 0 ? i + n : i;
        if (j < 0 || j >= n)
          return fail("Gather " + st.name + ": index " + std::to_string(i) + " out of range for " + std::to_string(n));
        idx.push_back(j);
      }
      y.shape = st.idx_rank == 0 ? std::vector<int64_t>{} : std::vector<int64_t>{(int64_t)idx.size()};
      y.hknown = x.hknown;
      y.hval.clear();
      if (x.hknown)
        for (int64_t j : idx) y.hval.push_back(x.hval[j]);
      return B200EP_OK;
    }
    case StepKind::kReduceSum: {
      if (x.shape.empty()) return fail("ReduceSum " + st.name + ": rank-0 data");
      y.shape = x.shape;
      if (st.keepdims) y.shape.back() = 1;
      else y.shape.pop_back();
      y.hknown = x.hknown;
      y.hval.clear();
      if (x.hknown) {
        const int64_t len = xs.back(), rows = len ? (int64_t)x.hval.size() / len : 0;
        for (int64_t r = 0; r < rows; ++r) {
          int64_t t = 0;
          for (int64_t c = 0; c < len; ++c) t = int_op(kOpAdd, t, x.hval[r * len + c], y.dtype);
          y.hval.push_back(t);
        }
      }
      return B200EP_OK;
    }
    case StepKind::kCopy: {
      std::vector<int64_t> o;
      if (st.layout == 1) {  // Unsqueeze: shape.rs:543-553
        const int64_t r = (int64_t)x.shape.size() + (int64_t)st.ivals.size();
        std::vector<char> ins(r, 0);
        for (int64_t a : st.ivals) {
          const int64_t k = a < 0 ? a + r : a;
          if (k < 0 || k >= r || ins[k]) return fail("Unsqueeze " + st.name + ": invalid axes");
          ins[k] = 1;
        }
        size_t j = 0;
        for (int64_t k = 0; k < r; ++k) o.push_back(ins[k] ? 1 : x.shape[j++]);
      } else if (st.layout == 2) {  // Squeeze: shape.rs:555-567
        const int64_t r = (int64_t)x.shape.size();
        std::vector<char> drop(r, 0);
        for (int64_t a : st.ivals) {
          const int64_t k = a < 0 ? a + r : a;
          if (k < 0 || k >= r || x.shape[k] != 1) return fail("Squeeze " + st.name + ": axis is not of extent 1");
          drop[k] = 1;
        }
        for (int64_t k = 0; k < r; ++k)
          if (!drop[k]) o.push_back(x.shape[k]);
      } else {  // Reshape with allowzero = 0: shape.rs:510-528
        int64_t known = 1, neg = -1;
        for (size_t k = 0; k < st.ivals.size(); ++k) {
          int64_t d = st.ivals[k];
          if (d == 0) {
            if (k >= x.shape.size()) return fail("Reshape " + st.name + ": 0 beyond the input rank");
            d = x.shape[k];
          }
          if (d == -1) {
            neg = (int64_t)k;
            o.push_back(1);
            continue;
          }
          known *= d;
          o.push_back(d);
        }
        const int64_t total = numel_of(x.shape);
        if (neg >= 0) {
          if (known == 0 || total % known) return fail("Reshape " + st.name + ": size does not divide");
          o[neg] = total / known;
        } else if (known != total) {
          return fail("Reshape " + st.name + ": element count changes");
        }
      }
      y.shape = o;
      y.hknown = x.hknown;
      y.hval = x.hknown ? x.hval : std::vector<int64_t>{};
      return B200EP_OK;
    }
    case StepKind::kBinary: {  // integer Add / Sub / Mul (the output shape is already set)
      const Slot& b = S[st.in[1]];
      y.hknown = x.hknown && b.hknown;
      y.hval.clear();
      if (!y.hknown) return B200EP_OK;
      const int rank = (int)y.shape.size();
      for (int64_t i = 0; i < numel_of(y.shape); ++i) {
        int64_t rem = i, ia = 0, ib = 0, sa = 1, sb = 1;
        for (int d = rank - 1; d >= 0; --d) {
          const int64_t c = rem % y.shape[d];
          rem /= y.shape[d];
          const int ja = (int)x.shape.size() - (rank - d), jb = (int)b.shape.size() - (rank - d);
          const int64_t da = ja >= 0 ? x.shape[ja] : 1, db = jb >= 0 ? b.shape[jb] : 1;
          if (da != 1) ia += c * sa;
          if (db != 1) ib += c * sb;
          sa *= da;
          sb *= db;
        }
        y.hval.push_back(int_op(st.bop, x.hval[ia], b.hval[ib], y.dtype));
      }
      return B200EP_OK;
    }
    case StepKind::kCast: {  // int32 <-> int64
      y.hknown = x.hknown;
      y.hval.clear();
      if (x.hknown)
        for (int64_t v : x.hval) y.hval.push_back(st.to == kI32 ? (int64_t)(int32_t)(uint32_t)(uint64_t)v : v);
      return B200EP_OK;
    }
    default:
      return B200EP_OK;
  }
}

int Plan::infer(std::vector<Slot>& S, std::string* err) const {
  auto fail = [&](const std::string& m) {
    *err = m;
    return B200EP_EINVAL;
  };
  seed_host_values(S);
  for (const Step& st : steps_) {
    switch (st.kind) {
      case StepKind::kShape:
      case StepKind::kGatherIdx:
      case StepKind::kReduceSum:
      case StepKind::kCopy:
        if (int rc = infer_glue(st, S, err)) return rc;
        break;
      case StepKind::kMnb: {
        if (st.pro) {  // the folded producer's outputs: its activation buffer and the residual
          auto sh = S[st.pro_x].shape;
          if (st.pro == kProSiluMul && !sh.empty()) sh.back() = st.pro_n;
          S[st.in[0]].shape = sh;
          if (st.pro_res >= 0) S[st.pro_res].shape = S[st.pro_x].shape;
        }
        const Slot& a = S[st.in[0]];
        if (a.shape.empty() || a.shape.back() != st.K)
          return fail("MatMulNBits " + st.name + ": input last dim " + shape_str(a.shape) + " != K=" + std::to_string(st.K));
        auto sh = a.shape;
        sh.back() = st.swiglu ? st.N / 2 : st.N;
        S[st.out[0]].shape = sh;
        if (st.swiglu && st.ws_slot >= 0) S[st.ws_slot].shape = {a.numel() / st.K * st.N};
        break;
      }
      case StepKind::kGqa: {
        const Slot& q = S[st.in[0]];
        const Slot& pk = S[st.in[3]];
        if (q.shape.size() != 3 || pk.shape.size() != 4)
          return fail("GroupQueryAttention " + st.name + ": query must be rank 3 and past_key rank 4");
        S[st.out[0]].shape = {q.shape[0], q.shape[1], (int64_t)st.num_heads * st.head_size};
        int64_t cap = pk.shape[2];
        // total_sequence_length when its value is known on the host (a host-resident input or
        // Cast(Gather(Shape(attention_mask), 1)) evaluated by the glue)
        const Slot& tot = S[st.in[6]];
        if (!st.sliding && tot.hknown && !tot.hval.empty()) cap = std::max<int64_t>(cap, tot.hval[0]);
        for (int o : {1, 2})
          if (st.out[o] >= 0 && S[st.out[o]].shape.empty())
            S[st.out[o]].shape = {pk.shape[0], pk.shape[1], cap, pk.shape[3]};
        break;
      }
      case StepKind::kPaged: {
        const Slot& q = S[st.in[0]];
        if (q.shape.size() != 2 || S[st.in[3]].shape.size() != 4)
          return fail("PagedAttention " + st.name + ": query must be rank 2 and key_cache rank 4");
        S[st.out[0]].shape = {q.shape[0], (int64_t)st.num_heads * st.head_size};
        for (int o : {1, 2})
          if (st.out[o] >= 0) S[st.out[o]].shape = S[st.in[o + 2]].shape;
        break;
      }
      case StepKind::kRms:
        S[st.out[0]].shape = S[st.in[0]].shape;
        if (st.skip && st.out[1] >= 0) S[st.out[1]].shape = S[st.in[0]].shape;
        break;
      case StepKind::kBinary: {
        const auto &a = S[st.in[0]].shape, &b = S[st.in[1]].shape;
        const size_t n = std::max(a.size(), b.size());
        std::vector<int64_t> o(n);
        for (size_t i = 0; i < n; ++i) {
          int64_t da = i < a.size() ? a[a.size() - 1 - i] : 1;
          int64_t db = i < b.size() ? b[b.size() - 1 - i] : 1;
          if (da != db && da != 1 && db != 1) return fail("binary " + st.name + ": shapes do not broadcast");
          o[n - 1 - i] = std::max(da, db);
        }
        S[st.out[0]].shape = o;
        if (is_int_dtype(S[st.out[0]].dtype))
          if (int rc = infer_glue(st, S, err)) return rc;
        break;
      }
      case StepKind::kSigmoid:
        S[st.out[0]].shape = S[st.in[0]].shape;
        break;
      case StepKind::kCast:
        S[st.out[0]].shape = S[st.in[0]].shape;
        if (is_int_dtype(st.to))
          if (int rc = infer_glue(st, S, err)) return rc;
        break;
      case StepKind::kSiluMul: {
        auto sh = S[st.in[0]].shape;
        sh.back() = st.N;
        S[st.out[0]].shape = sh;
        break;
      }
      case StepKind::kGbq: {
        auto sh = S[st.in[0]].shape;
        sh.push_back(st.gbq_dim);
        S[st.out[0]].shape = sh;
        break;
      }
      case StepKind::kAllReduce:
        S[st.out[0]].shape = S[st.in[0]].shape;
        break;
      case StepKind::kAllGather: {
        auto sh = S[st.in[0]].shape;
        sh.back() = st.N;
        S[st.out[0]].shape = sh;
        if (st.ws_slot >= 0) S[st.ws_slot].shape = {S[st.in[0]].numel() * (st.N / std::max<int64_t>(st.shard_cols, 1))};
        break;
      }
    }
  }
  return B200EP_OK;
}

int Plan::output_shapes(const std::vector<TensorArg>& in, std::vector<std::vector<int64_t>>* shapes) {
  std::lock_guard<std::mutex> lk(mu_);
  if (in.size() != in_names_.size())
    return set_error(B200EP_EINVAL, "expected " + std::to_string(in_names_.size()) + " inputs, got " +
                                        std::to_string(in.size()));
  std::vector<Slot> S = slots_;
  for (auto& s : S) {
    if (s.kind == Slot::kInput) {
      s.shape = in[s.io].shape;
      if (!in[s.io].on_device && in[s.io].data && numel_of(s.shape) == 1 && dtype_size(s.dtype) <= 8) {
        s.host_copy.resize(dtype_size(s.dtype));
        memcpy(s.host_copy.data(), in[s.io].data, s.host_copy.size());
      }
    } else if (s.kind != Slot::kConst) {
      s.shape.clear();
    }
  }
  std::string err;
  if (infer(S, &err)) return set_error(B200EP_EINVAL, err);
  shapes->assign(out_names_.size(), {});
  for (auto& s : S)
    if (s.kind == Slot::kOutput) (*shapes)[s.io] = s.shape;
  return B200EP_OK;
}

// ---- launches -------------------------------------------------------------------------------
int Plan::launch_steps(const std::vector<Slot>& S, Program& prog, cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(st, &cs);
  const bool prof = prof_ && cs == cudaStreamCaptureStatusNone;
  if (prof && prof_ev_.size() < 2 * steps_.size() + 2) {
    for (auto ev : prof_ev_) cudaEventDestroy(ev);
    prof_ev_.assign(2 * steps_.size() + 2, nullptr);
    for (auto& ev : prof_ev_) cudaEventCreate(&ev);
  }
  // the attention kernels read their lengths / block tables before their programmatic-launch
  // wait (data written two or more kernels back); when the step launched just before produced
  // one of them (integer glue right in front of the attention), that launch serialises fully
  std::vector<int> producer(S.size(), -1);
  for (int i = 0; i < (int)steps_.size(); ++i)
    for (int o : steps_[i].out)
      if (o >= 0) producer[o] = i;
  int prev_launch = -1;
  int si = 0;
  for (const Step& s : steps_) {
    if (prof) cudaEventRecord(prof_ev_[2 * si], st);
    ++si;
    cudaError_t e = cudaSuccess;
    if (!prog.host_step.empty() && prog.host_step[si - 1]) {  // evaluated on the host, value uploaded
      if (prof) cudaEventRecord(prof_ev_[2 * si - 1], st);
      continue;
    }
    bool fresh = false;
    if (s.kind == StepKind::kGqa || s.kind == StepKind::kPaged)
      for (int k = 5; k <= 7 && k < (int)s.in.size(); ++k)
        fresh |= s.in[k] >= 0 && prev_launch >= 0 && producer[s.in[k]] == prev_launch;
    std::unique_ptr<PdlOff> pdl_off(fresh ? new PdlOff() : nullptr);
    prev_launch = si - 1;
    switch (s.kind) {
      case StepKind::kMnb: {
        const Slot& a = S[s.in[0]];
        if (s.prepacked) {
          MnbPacked pk = mnb_packed_geometry(s.N, s.K, s.block);
          pk.w = s.pk_w->p;
          const int64_t M = a.numel() / s.K;
          MnbAr oar;
          if (s.ar_out && ar_fused(M, s.N, s.ar_block)) oar = make_ar(*cfg_.tp);
          const MnbAr* out_ar = oar.world ? &oar : nullptr;
          if (s.pro) {
            MnbPro pro;
            pro.kind = s.pro;
            pro.x = S[s.pro_x].ptr;
            pro.skip = s.pro_skip >= 0 ? S[s.pro_skip].ptr : nullptr;
            pro.gamma = s.pro_gamma >= 0 ? S[s.pro_gamma].ptr : nullptr;
            pro.residual = s.pro_res >= 0 ? S[s.pro_res].ptr : nullptr;
            pro.eps = s.pro_eps;
            pro.swiglu = s.swiglu ? 1 : 0;
            if (s.pro_ar && ar_fused(M, s.K, s.block)) pro.ar = make_ar(*cfg_.tp);
            bool aligned = true;
            for (const void* q : {pro.x, pro.skip, pro.gamma, (const void*)pro.residual})
              aligned &= (reinterpret_cast<uintptr_t>(q) & 15) == 0;
            if (aligned && mnb_prologue_fits(M, s.K, s.block)) {
              e = launch_mnb_packed(nullptr, pk, S[s.out[0]].ptr, a.dtype, M, st, &pro, out_ar);
              break;
            }
            // rows too large to stage (prefill): the standalone producer, then the plain GEMV
            if (s.pro == kProSiluMul) {
              e = launch_silu_mul(pro.x, a.ptr, a.dtype, M, s.pro_n, st);
            } else {
              RmsArgs r{pro.x, pro.skip, pro.gamma, a.ptr, pro.residual, a.dtype, M, s.K, s.pro_eps};
              e = launch_rms_norm(r, st);
            }
            if (e != cudaSuccess) break;
          }
          MnbPro epi;  // no prologue; the SwiGLU epilogue when the rows are interleaved
          epi.swiglu = s.swiglu ? 1 : 0;
          if (!out_ar && mnb_gemm_supported(M, s.K, a.ptr)) {
            // prefill rows: the GEMM writes gate and up (interleaved) into the workspace first
            void* y = s.swiglu ? S[s.ws_slot].ptr : S[s.out[0]].ptr;
            e = launch_mnb_gemm(a.ptr, pk, y, a.dtype, M, st);
            if (e == cudaSuccess && s.swiglu) e = launch_silu_mul_interleaved(y, S[s.out[0]].ptr, a.dtype, M, s.N / 2, st);
          } else {
            e = launch_mnb_packed(a.ptr, pk, S[s.out[0]].ptr, a.dtype, M, st, &epi, out_ar);
          }
          break;
        }
        void* y = s.swiglu ? S[s.ws_slot].ptr : S[s.out[0]].ptr;
        MnbArgs m{a.ptr, static_cast<const uint8_t*>(S[s.wB].ptr), S[s.wS].ptr,
                  s.wZ >= 0 ? static_cast<const uint8_t*>(S[s.wZ].ptr) : nullptr,
                  y, a.dtype, a.numel() / s.K, s.N, s.K, s.bits, s.block};
        e = launch_matmulnbits(m, st);
        if (e == cudaSuccess && s.swiglu)
          e = launch_silu_mul_interleaved(y, S[s.out[0]].ptr, a.dtype, a.numel() / s.K, s.N / 2, st);
        break;
      }
      case StepKind::kGqa: {
        const Slot& q = S[s.in[0]];
        const Slot& past_k = S[s.in[3]];
        const Slot& past_v = S[s.in[4]];
        const Slot& pres_k = S[s.out[1]];
        const Slot& pres_v = S[s.out[2]];
        const int64_t B = q.shape[0], Sq = q.shape[1];
        const int64_t pcap = past_k.shape[2], cap = pres_k.shape[2];
        const int esz = dtype_size(q.dtype);
        if (s.sliding) {
          // the sliding-window cache: rows reclaimed from the front, present written from row 0
          const Slot* cos = s.in[7] >= 0 ? &S[s.in[7]] : nullptr;
          GqaSlidingArgs a{};
          a.p.batch = B;
          a.p.seq = Sq;
          a.p.num_heads = s.num_heads;
          a.p.kv_heads = s.kv_heads;
          a.p.head_size = s.head_size;
          a.p.cap = pcap;
          a.p.do_rotary = s.do_rotary && cos;
          a.p.max_seq = cos ? cos->shape[0] : 0;
          a.p.rotary_half = cos ? cos->shape[1] : 0;
          a.p.interleaved = s.interleaved;
          a.p.packed_qkv = s.packed;
          a.p.local_window = s.local_window;
          a.p.scale = s.scale;
          a.query = q.ptr;
          a.key = s.packed ? nullptr : S[s.in[1]].ptr;
          a.value = s.packed ? nullptr : S[s.in[2]].ptr;
          a.past_key = past_k.ptr;
          a.past_value = past_v.ptr;
          a.present_key = pres_k.ptr;
          a.present_value = pres_v.ptr;
          a.seqlens_k = static_cast<const int32_t*>(S[s.in[5]].ptr);
          a.cos_cache = cos ? cos->ptr : nullptr;
          a.sin_cache = s.in[8] >= 0 ? S[s.in[8]].ptr : nullptr;
          a.out = S[s.out[0]].ptr;
          a.dtype = q.dtype;
          a.workspace = S[s.ws_slot].ptr;
          a.workspace_bytes = (size_t)S[s.ws_slot].numel();
          if (int rc = launch_gqa_sliding(a, st)) return rc;
          break;
        }
        if (pres_k.ptr != past_k.ptr || pres_v.ptr != past_v.ptr) {
          // growing contract: present = past rows followed by the new rows
          const int64_t rows = std::min(pcap, cap);
          const size_t row_bytes = (size_t)s.head_size * esz;
          for (auto [dst, src] : {std::pair<void*, void*>{pres_k.ptr, past_k.ptr}, {pres_v.ptr, past_v.ptr}}) {
            if (rows > 0) {
              e = cudaMemcpy2DAsync(dst, cap * row_bytes, src, pcap * row_bytes, rows * row_bytes,
                                    B * s.kv_heads, cudaMemcpyDeviceToDevice, st);
              if (e != cudaSuccess) return cuda_status(e, "GroupQueryAttention present copy");
            }
          }
        }
        GqaArgs a{};
        a.p.batch = B;
        a.p.seq = Sq;
        a.p.num_heads = s.num_heads;
        a.p.kv_heads = s.kv_heads;
        a.p.head_size = s.head_size;
        a.p.cap = cap;
        const Slot* cos = s.in[7] >= 0 ? &S[s.in[7]] : nullptr;
        a.p.do_rotary = s.do_rotary && cos;
        a.p.max_seq = cos ? cos->shape[0] : 0;
        a.p.rotary_half = cos ? cos->shape[1] : 0;
        a.p.interleaved = s.interleaved;
        a.p.packed_qkv = s.packed;
        a.p.local_window = s.local_window;
        a.p.scale = s.scale;
        a.p.qk_norm_eps = s.qk_eps;
        if (s.in[10] >= 0) {
          a.p.bias_batch = S[s.in[10]].shape[0];
          a.p.bias_total = S[s.in[10]].shape[3];
          a.bias = S[s.in[10]].ptr;
        }
        a.query = q.ptr;
        a.key = s.packed ? nullptr : S[s.in[1]].ptr;
        a.value = s.packed ? nullptr : S[s.in[2]].ptr;
        a.kv_key = pres_k.ptr;
        a.kv_value = pres_v.ptr;
        a.seqlens_k = static_cast<const int32_t*>(S[s.in[5]].ptr);
        a.cos_cache = cos ? cos->ptr : nullptr;
        a.sin_cache = s.in[8] >= 0 ? S[s.in[8]].ptr : nullptr;
        a.q_norm = s.in[14] >= 0 ? S[s.in[14]].ptr : nullptr;
        a.k_norm = s.in[15] >= 0 ? S[s.in[15]].ptr : nullptr;
        a.out = S[s.out[0]].ptr;
        a.dtype = q.dtype;
        a.workspace = S[s.ws_slot].ptr;
        a.workspace_bytes = (size_t)S[s.ws_slot].numel();
        int rc = launch_gqa(a, st);
        if (rc) return rc;
        break;
      }
      case StepKind::kPaged: {
        const Slot& q = S[s.in[0]];
        const Slot& kc_in = S[s.in[3]];
        const Slot& vc_in = S[s.in[4]];
        // the caches are updated where the outputs live: copied there first when ORT bound the
        // outputs apart from the inputs, else the inputs themselves (the reference's write-back)
        void* kc = s.out[1] >= 0 ? S[s.out[1]].ptr : kc_in.ptr;
        void* vc = s.out[2] >= 0 ? S[s.out[2]].ptr : vc_in.ptr;
        for (auto [dst, src] : {std::pair<void*, const Slot*>{kc, &kc_in}, {vc, &vc_in}})
          if (dst != src->ptr) {
            e = cudaMemcpyAsync(dst, src->ptr, (size_t)src->numel() * dtype_size(src->dtype), cudaMemcpyDeviceToDevice, st);
            if (e != cudaSuccess) return cuda_status(e, "PagedAttention cache copy");
          }
        b200ep_paged_params p{};
        p.batch = (int32_t)(S[s.in[5]].numel() - 1);
        p.num_tokens = (int32_t)q.shape[0];
        p.num_heads = s.num_heads;
        p.kv_heads = s.kv_heads;
        p.head_size = s.head_size;
        p.num_blocks = (int32_t)kc_in.shape[0];
        p.block_size = (int32_t)kc_in.shape[1];
        p.max_blocks = p.batch > 0 ? (int32_t)(S[s.in[7]].numel() / p.batch) : 0;
        const Slot* cos = s.do_rotary && s.in[8] >= 0 ? &S[s.in[8]] : nullptr;
        p.do_rotary = cos != nullptr;
        p.max_seq = cos ? (int32_t)cos->shape[0] : 0;
        p.rotary_half = cos ? (int32_t)cos->shape[1] : 0;
        p.interleaved = s.interleaved;
        p.scale = s.scale;
        int rc = b200ep_paged_attention(&p, q.ptr, S[s.in[1]].ptr, S[s.in[2]].ptr, kc, vc,
                                        static_cast<const int32_t*>(S[s.in[5]].ptr),
                                        static_cast<const int32_t*>(S[s.in[6]].ptr),
                                        static_cast<const int32_t*>(S[s.in[7]].ptr), cos ? cos->ptr : nullptr,
                                        cos ? S[s.in[9]].ptr : nullptr, S[s.out[0]].ptr, q.dtype, st);
        if (rc) return rc;
        break;
      }
      case StepKind::kRms: {
        const Slot& x = S[s.in[0]];
        const int64_t hidden = x.shape.back();
        RmsArgs r{x.ptr, s.skip ? S[s.in[1]].ptr : nullptr, S[s.in[s.skip ? 2 : 1]].ptr, S[s.out[0]].ptr,
                  s.skip && s.out[1] >= 0 ? S[s.out[1]].ptr : nullptr, x.dtype, x.numel() / hidden, hidden, s.eps};
        e = launch_rms_norm(r, st);
        break;
      }
      case StepKind::kBinary: {
        const Slot &a = S[s.in[0]], &b = S[s.in[1]], &y = S[s.out[0]];
        BinaryGeom gm;
        gm.rank = (int)y.shape.size();
        gm.total = y.numel();
        int64_t sa = 1, sb = 1;
        for (int d = gm.rank - 1; d >= 0; --d) {
          gm.out_dims[d] = y.shape[d];
          const int ia = (int)a.shape.size() - (gm.rank - d), ib = (int)b.shape.size() - (gm.rank - d);
          const int64_t da = ia >= 0 ? a.shape[ia] : 1, db = ib >= 0 ? b.shape[ib] : 1;
          gm.a_strides[d] = da == 1 ? 0 : sa;
          gm.b_strides[d] = db == 1 ? 0 : sb;
          sa *= da;
          sb *= db;
        }
        e = is_int_dtype(y.dtype) ? launch_binary_int(a.ptr, b.ptr, y.ptr, y.dtype, gm, s.bop, st)
                                  : launch_binary(a.ptr, b.ptr, y.ptr, y.dtype, gm, s.bop, st);
        break;
      }
      case StepKind::kShape:  // always known on the host
        break;
      case StepKind::kGatherIdx: {
        const Slot& x = S[s.in[0]];
        IdxList il;
        il.n = (int)s.ivals.size();
        for (int i = 0; i < il.n; ++i) il.v[i] = s.ivals[i] < 0 ? s.ivals[i] + x.shape[0] : s.ivals[i];
        e = launch_gather_idx(x.ptr, S[s.out[0]].ptr, x.dtype, il, st);
        break;
      }
      case StepKind::kReduceSum: {
        const Slot& x = S[s.in[0]];
        auto d = prog.dims_idx.find(s.in[0]);
        const int64_t len = x.shape.back();
        e = launch_reduce_sum_rows(x.ptr, x.dtype, S[s.out[0]].ptr, S[s.out[0]].dtype, len ? x.numel() / len : 0, len,
                                   d == prog.dims_idx.end() ? nullptr : prog.dims_dev + d->second, st);
        break;
      }
      case StepKind::kCopy: {
        const Slot& x = S[s.in[0]];
        e = launch_copy_bytes(x.ptr, S[s.out[0]].ptr, x.numel() * dtype_size(x.dtype), st);
        break;
      }
      case StepKind::kSigmoid:
        e = launch_sigmoid(S[s.in[0]].ptr, S[s.out[0]].ptr, S[s.in[0]].dtype, S[s.in[0]].numel(), st);
        break;
      case StepKind::kSiluMul: {
        const Slot& gu = S[s.in[0]];
        e = launch_silu_mul(gu.ptr, S[s.out[0]].ptr, gu.dtype, gu.numel() / (2 * s.N), s.N, st);
        break;
      }
      case StepKind::kCast:
        e = is_int_dtype(s.to) ? launch_cast_int(S[s.in[0]].ptr, S[s.in[0]].dtype, S[s.out[0]].ptr, s.to,
                                                 S[s.in[0]].numel(), st)
                               : launch_cast(S[s.in[0]].ptr, S[s.in[0]].dtype, S[s.out[0]].ptr, s.to,
                                             S[s.in[0]].numel(), st);
        break;
      case StepKind::kGbq: {
        const Slot& idx = S[s.in[0]];
        GbqArgs a{static_cast<const uint8_t*>(S[s.wB].ptr), S[s.wS].ptr,
                  s.wZ >= 0 ? static_cast<const uint8_t*>(S[s.wZ].ptr) : nullptr, idx.ptr, idx.dtype,
                  S[s.out[0]].ptr, S[s.out[0]].dtype, idx.numel(), s.gbq_rows, s.gbq_dim, s.block,
                  device_error_slot()};
        e = launch_gather_block_quantized(a, st);
        break;
      }
      case StepKind::kAllReduce:
      case StepKind::kAllGather: {
        if (s.ar_skip) {
          const Slot& x = S[s.in[0]];
          const int64_t hidden = x.shape.back();
          if (ar_fused(x.numel() / hidden, hidden, s.ar_block)) break;  // summed in the consumer's prologue
        }
        int rc = tp_collective(*cfg_.tp, s, S, st);
        if (rc) return rc;
        break;
      }
    }
    if (e != cudaSuccess) return cuda_status(e, ("launch " + s.name).c_str());
    if (prof) cudaEventRecord(prof_ev_[2 * si - 1], st);
  }
  if (prof) {
    cudaStreamSynchronize(st);
    for (int i = 0; i < si; ++i) {
      const Step& s = steps_[i];
      std::string key = step_kind_name(s.kind);
      if (s.kind == StepKind::kMnb)
        key += " M=" + std::to_string(S[s.in[0]].numel() / std::max<int64_t>(s.K, 1)) + " N=" + std::to_string(s.N) +
               " K=" + std::to_string(s.K) + (s.pro ? " +prologue" : "") + (s.ar_out ? " +peer-out" : "");
      else if (s.kind == StepKind::kGqa)
        key += " rows=" + std::to_string(S[s.in[0]].numel() / std::max<int64_t>(S[s.in[0]].shape.back(), 1));
      float ms = 0.f;
      cudaEventElapsedTime(&ms, prof_ev_[2 * i], prof_ev_[2 * i + 1]);
      auto& v = prof_ms_[key];
      v.first += 1;
      v.second += ms;
    }
  }
  return B200EP_OK;
}

int Plan::launches_per_run() const {
  int n = 0;
  for (auto& s : steps_)
    n += (s.kind != StepKind::kAllReduce && s.kind != StepKind::kAllGather && s.kind != StepKind::kShape) +
         (s.kind == StepKind::kPaged);
  return n;
}

// ---- inputs whose key axis changes every call ----------------------------------------------
void Plan::compute_free_rules() {
  free_rule_.assign(in_names_.size(), 0);
  Uses u = uses_of(steps_, slots_.size());
  for (size_t id = 0; id < slots_.size(); ++id) {
    const Slot& sl = slots_[id];
    if (sl.kind != Slot::kInput) continue;
    bool folded = false;  // read by a GEMV prologue: never free
    for (const Step& st : steps_)
      for (int x : {st.pro_x, st.pro_skip, st.pro_gamma, st.pro_res})
        folded |= x == (int)id;
    const auto& users = u.users[id];
    if (folded || users.empty()) continue;
    bool shape_only = true, reducible = true;
    for (int k : users) {
      const StepKind kd = steps_[k].kind;
      shape_only &= kd == StepKind::kShape;
      reducible &= kd == StepKind::kShape || (kd == StepKind::kReduceSum && steps_[k].in[0] == (int)id);
    }
    free_rule_[sl.io] = shape_only ? 1 : reducible ? 2 : 0;
  }
}

std::vector<int64_t> Plan::key_shape(int io, const std::vector<int64_t>& shape) const {
  const int rule = io < (int)free_rule_.size() ? free_rule_[io] : 0;
  if (rule == 0 || shape.empty()) return shape;
  std::vector<int64_t> k = shape;
  if (rule == 1) {
    std::fill(k.begin(), k.end(), 1);
  } else {
    int64_t c = 64;
    while (c < shape.back()) c *= 2;
    k.back() = c;
  }
  return k;
}

int Plan::stage_dynamic(Program& prog, const std::vector<TensorArg>& in, cudaStream_t st) {
  std::vector<Slot>& S = prog.slots;
  bool dims = false;
  for (size_t id = 0; id < S.size(); ++id) {
    Slot& s = S[id];
    if (s.kind != Slot::kInput || free_rule_[s.io] == 0) continue;
    const TensorArg& a = in[s.io];
    s.rshape = a.shape;
    if (free_rule_[s.io] != 2) continue;
    const size_t bytes = (size_t)numel_of(a.shape) * dtype_size(s.dtype);
    if (bytes) {
      B200EP_CUDA_RET(cudaMemcpyAsync(s.ptr, a.data, bytes, a.on_device ? cudaMemcpyDeviceToDevice
                                                                       : cudaMemcpyHostToDevice, st));
    }
    prog.dims_host[prog.dims_idx.at((int)id)] = a.shape.back();
    dims = true;
  }
  if (dims)
    B200EP_CUDA_RET(cudaMemcpyAsync(prog.dims_dev, prog.dims_host.data(), prog.dims_host.size() * 8,
                                    cudaMemcpyHostToDevice, st));
  if (prog.host_steps.empty()) return B200EP_OK;
  // re-evaluate the host-side glue for this call (shapes of changing inputs, host scalars)
  for (auto& s : S)
    if (s.kind == Slot::kInput && is_int_dtype(s.dtype) && !s.host_copy.empty()) s.hval = ints_of(s.host_copy, s.dtype);
  std::string err;
  for (int i : prog.host_steps)
    if (infer_glue(steps_[i], S, &err)) return set_error(B200EP_EINVAL, err);
  auto pack = [&](const Slot& s, uint8_t* dst) {
    for (size_t k = 0; k < s.hval.size(); ++k) {
      if (s.dtype == kI32) {
        const int32_t v = (int32_t)s.hval[k];
        memcpy(dst + 4 * k, &v, 4);
      } else {
        memcpy(dst + 8 * k, &s.hval[k], 8);
      }
    }
  };
  for (auto [id, off] : prog.uploads) pack(S[id], prog.upl_host.data() + off);
  if (!prog.upl_host.empty())
    B200EP_CUDA_RET(cudaMemcpyAsync(prog.upl_dev, prog.upl_host.data(), prog.upl_host.size(), cudaMemcpyHostToDevice, st));
  for (int id : prog.out_uploads) {
    const Slot& s = S[id];
    std::vector<uint8_t> tmp(s.hval.size() * dtype_size(s.dtype));
    pack(s, tmp.data());
    if (!tmp.empty()) B200EP_CUDA_RET(cudaMemcpyAsync(s.ptr, tmp.data(), tmp.size(), cudaMemcpyHostToDevice, st));
  }
  // a total_sequence_length computed from this call's mask must fit the compiled cache capacity
  for (const Step& stp : steps_)
    if (stp.kind == StepKind::kGqa && !stp.sliding && stp.in[6] >= 0) {
      const Slot& tot = S[stp.in[6]];
      const int64_t cap = S[stp.out[1]].shape.size() == 4 ? S[stp.out[1]].shape[2] : 0;
      if (tot.hknown && !tot.hval.empty() && tot.hval[0] > cap)
        return set_error(B200EP_EINVAL, "GroupQueryAttention " + stp.name + ": total_sequence_length " +
                                            std::to_string(tot.hval[0]) + " exceeds the KV capacity " +
                                            std::to_string(cap));
    }
  return B200EP_OK;
}

int Plan::run(const std::vector<TensorArg>& in, const std::vector<TensorArg>& out, cudaStream_t caller) {
  std::lock_guard<std::mutex> lk(mu_);
  // Work runs on the plan's own stream (capturable even when the caller uses the legacy
  // stream), ordered after the caller's prior work and before its later work by two events.
  if (!stream_) {
    B200EP_CUDA_RET(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    B200EP_CUDA_RET(cudaEventCreateWithFlags(&ev_in_, cudaEventDisableTiming));
    B200EP_CUDA_RET(cudaEventCreateWithFlags(&ev_out_, cudaEventDisableTiming));
  }
  cudaStream_t st = stream_;
  B200EP_CUDA_RET(cudaEventRecord(ev_in_, caller));
  B200EP_CUDA_RET(cudaStreamWaitEvent(st, ev_in_, 0));
  const auto t0 = std::chrono::steady_clock::now();
  int rc = run_locked(in, out, st);
  if (cfg_.summary) {
    std::lock_guard<std::mutex> sl(cfg_.summary->mu);
    cfg_.summary->run_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  }
  cudaEventRecord(ev_out_, st);
  cudaStreamWaitEvent(caller, ev_out_, 0);
  return rc;
}

int Plan::run_locked(const std::vector<TensorArg>& in, const std::vector<TensorArg>& out, cudaStream_t st) {
  if (in.size() != in_names_.size() || out.size() != out_names_.size())
    return set_error(B200EP_EINVAL, "run: expected " + std::to_string(in_names_.size()) + " inputs and " +
                                        std::to_string(out_names_.size()) + " outputs");
  // Repeat of the previous call (same pointers, residency and shapes): replay its graph directly,
  // skipping the shape-key and pointer-key lookups (they cost tens of microseconds per call).
  if (free_rule_.size() != in_names_.size()) free_rule_.assign(in_names_.size(), 0);
  // (inputs with a changing key axis enter by their key shape and are always copied in)
  std::vector<int64_t> sig;
  sig.reserve(4 * (in.size() + out.size()) + 2);
  for (const auto* v : {&in, &out}) {
    sig.push_back((int64_t)v->size());
    for (size_t i = 0; i < v->size(); ++i) {
      const TensorArg& a = (*v)[i];
      const bool free_in = v == &in && free_rule_[i] != 0;
      sig.push_back(free_in ? 0 : (int64_t)reinterpret_cast<uintptr_t>(a.data));
      sig.push_back(a.on_device ? 1 : 0);
      sig.push_back((int64_t)a.shape.size());
      const std::vector<int64_t> ks = free_in ? key_shape((int)i, a.shape) : a.shape;
      sig.insert(sig.end(), ks.begin(), ks.end());
    }
  }
  if (last_prog_ && last_exec_ && sig == last_sig_) {
    Program& prog = *last_prog_;
    std::vector<Slot>& S = prog.slots;
    int64_t h2d = 0, d2h = 0;
    for (auto& s : S)
      if (s.kind == Slot::kInput && !in[s.io].on_device && free_rule_[s.io] == 0) {
        const size_t bytes = (size_t)numel_of(s.shape) * dtype_size(s.dtype);
        if (bytes) B200EP_CUDA_RET(cudaMemcpyAsync(s.ptr, in[s.io].data, bytes, cudaMemcpyHostToDevice, st));
        if (!s.host_copy.empty()) memcpy(s.host_copy.data(), in[s.io].data, s.host_copy.size());
        h2d += (int64_t)bytes;
      }
    if (int rc = stage_dynamic(prog, in, st)) return rc;
    ++stats_.runs;
    B200EP_CUDA_RET(cudaGraphLaunch(last_exec_, st));
    ++stats_.graph_replays;
    bool any_host_out = false;
    for (auto& s : S)
      if (s.kind == Slot::kOutput && !out[s.io].on_device) {
        const size_t bytes = (size_t)numel_of(s.shape) * dtype_size(s.dtype);
        if (bytes) B200EP_CUDA_RET(cudaMemcpyAsync(out[s.io].data, s.ptr, bytes, cudaMemcpyDeviceToHost, st));
        d2h += (int64_t)bytes;
        any_host_out = true;
      }
    if (SessionSummary* sum = cfg_.summary.get()) {
      std::lock_guard<std::mutex> sl(sum->mu);
      ++sum->key_hits;
      ++(prog.path == 0 ? sum->path_decode : prog.path == 1 ? sum->path_prefill : sum->path_general);
      ++sum->graph_replays;
      sum->h2d_bytes += h2d;
      sum->d2h_bytes += d2h;
    }
    if (any_host_out) B200EP_CUDA_RET(cudaStreamSynchronize(st));
    return B200EP_OK;
  }
  last_prog_ = nullptr;
  last_exec_ = nullptr;
  // shape key: input shapes plus which inputs are host-resident
  std::string key;
  for (size_t i = 0; i < in.size(); ++i)
    key += shape_str(key_shape((int)i, in[i].shape)) + (free_rule_[i] == 1 ? "x" : in[i].on_device ? "d" : "h") + ";";
  for (size_t i = 0; i < out.size(); ++i) key += shape_str(out[i].shape) + (out[i].on_device ? "d" : "h") + ";";
  auto it = programs_.find(key);
  SessionSummary* sum = cfg_.summary.get();
  if (sum) {
    std::lock_guard<std::mutex> sl(sum->mu);
    ++(it == programs_.end() ? sum->key_misses : sum->key_hits);
  }
  if (it == programs_.end()) {
    auto prog = std::make_unique<Program>();
    prog->slots = slots_;
    for (auto& s : prog->slots) {
      if (s.kind == Slot::kInput) {
        s.shape = key_shape(s.io, in[s.io].shape);
        if (free_rule_[s.io]) s.rshape = in[s.io].shape;
        if (in[s.io].dtype != s.dtype && s.dtype != 0)
          return set_error(B200EP_EINVAL, "input " + s.name + " has dtype " + std::to_string(in[s.io].dtype) +
                                              ", expected " + std::to_string(s.dtype));
        s.dtype = in[s.io].dtype;
        if (!in[s.io].on_device && !free_rule_[s.io] && numel_of(s.shape) == 1 && dtype_size(s.dtype) <= 8) {
          s.host_copy.resize(dtype_size(s.dtype));
          memcpy(s.host_copy.data(), in[s.io].data, s.host_copy.size());
        }
      } else if (s.kind == Slot::kOutput) {
        s.shape = out[s.io].shape;  // caller-provided (authoritative for present buffers)
      } else if (s.kind != Slot::kConst) {
        s.shape.clear();
      }
    }
    std::string err;
    if (infer(prog->slots, &err)) return set_error(B200EP_EINVAL, err);
    for (auto& s : prog->slots)
      if (s.kind == Slot::kOutput && s.shape != out[s.io].shape)
        return set_error(B200EP_EINVAL, "output " + s.name + " bound with shape " + shape_str(out[s.io].shape) +
                                            ", plan computes " + shape_str(s.shape));
    // integer glue whose values infer computed on the host: no launch; device readers of those
    // values get them from one packed upload per call
    prog->host_step.assign(steps_.size(), 0);
    std::vector<char> dev_read(prog->slots.size(), 0);
    for (size_t i = 0; i < steps_.size(); ++i) {
      const Step& stp = steps_[i];
      const bool glue = stp.kind == StepKind::kShape || stp.kind == StepKind::kGatherIdx ||
                        stp.kind == StepKind::kReduceSum || stp.kind == StepKind::kCopy ||
                        ((stp.kind == StepKind::kBinary || stp.kind == StepKind::kCast) &&
                         is_int_dtype(prog->slots[stp.out[0]].dtype));
      if (glue && prog->slots[stp.out[0]].hknown) {
        prog->host_step[i] = 1;
        prog->host_steps.push_back((int)i);
        continue;
      }
      for (int id : stp.in)
        if (id >= 0) dev_read[id] = 1;
      for (int id : {stp.pro_x, stp.pro_skip, stp.pro_gamma})
        if (id >= 0) dev_read[id] = 1;
    }
    size_t upl_bytes = 0;
    for (size_t id = 0; id < prog->slots.size(); ++id) {
      const Slot& sl = prog->slots[id];
      if (!sl.hknown || sl.kind == Slot::kConst || sl.kind == Slot::kInput) continue;
      if (sl.kind == Slot::kOutput) {
        prog->out_uploads.push_back((int)id);
      } else if (dev_read[id]) {
        prog->uploads.push_back({(int)id, upl_bytes});
        upl_bytes += ((size_t)std::max<int64_t>(numel_of(sl.shape), 1) * dtype_size(sl.dtype) + 15) & ~(size_t)15;
      }
    }
    prog->upl_host.assign(upl_bytes, 0);
    for (size_t id = 0; id < prog->slots.size(); ++id) {
      const Slot& sl = prog->slots[id];
      if (sl.kind == Slot::kInput && free_rule_[sl.io] == 2) {
        const int k = (int)prog->dims_idx.size();
        prog->dims_idx[(int)id] = k;
      }
    }
    prog->dims_host.assign(prog->dims_idx.size(), 0);
    // workspaces for attention steps: the steps run one after another on one stream, so steps of
    // the same kind (plain / sliding-window cache) and KV geometry share one zero-filled workspace
    // (the kernels leave its counters zeroed), sized for the largest of them
    std::map<std::tuple<bool, int64_t, int64_t>, int> ws_of;
    for (Step& stp : steps_)
      if (stp.kind == StepKind::kGqa && stp.ws_slot < 0) {
        const Slot& q = prog->slots[stp.in[0]];
        const auto key = std::make_tuple(stp.sliding, q.shape.empty() ? 0 : q.shape[0], (int64_t)stp.kv_heads);
        auto f = ws_of.find(key);
        if (f != ws_of.end()) {
          stp.ws_slot = f->second;
          continue;
        }
        Slot w;
        w.name = stp.name + "#ws";
        w.dtype = kU8;
        stp.ws_slot = (int)slots_.size();
        ws_of[key] = stp.ws_slot;
        slots_.push_back(w);
        prog->slots.push_back(w);
      }
    for (Step& stp : steps_)
      if (stp.kind == StepKind::kGqa) {
        const Slot& q = prog->slots[stp.in[0]];
        b200ep_gqa_params p{};
        p.batch = q.shape[0];
        p.seq = q.shape[1];
        p.num_heads = stp.num_heads;
        p.kv_heads = stp.kv_heads;
        p.head_size = stp.head_size;
        p.cap = prog->slots[stp.out[1]].shape[2];
        p.local_window = stp.local_window;
        const int64_t need = (int64_t)(stp.sliding ? gqa_sliding_workspace_bytes(p, q.dtype) : gqa_workspace_bytes(p));
        auto& sh = prog->slots[stp.ws_slot].shape;
        if (sh.empty() || sh[0] < need) sh = {need};
      }
    // allocate: zero-filled workspaces and host staging each get their own buffer; the other
    // temporaries share one arena by lifetime (first to last step that touches them), so a deep
    // prefill does not hold every layer's activations at once.  Reuse is safe under programmatic
    // dependent launch: a kernel writes its outputs only after its pdl_wait, when every earlier
    // kernel — and so every earlier reader of a reused buffer — has completed.
    const int nst = (int)steps_.size();
    std::vector<int> first(prog->slots.size(), nst), last(prog->slots.size(), -1);
    for (int si = 0; si < nst; ++si) {
      const Step& st = steps_[si];
      auto touch = [&](int id) {
        if (id < 0 || id >= (int)prog->slots.size()) return;
        first[id] = std::min(first[id], si);
        last[id] = std::max(last[id], si);
      };
      for (int id : st.in) touch(id);
      for (int id : st.out) touch(id);
      for (int id : {st.pro_x, st.pro_skip, st.pro_gamma, st.pro_res, st.ws_slot}) touch(id);
    }
    struct Place {
      int id;
      size_t bytes, off;
    };
    std::vector<Place> arena;
    std::vector<char> uploaded(prog->slots.size(), 0);
    for (auto [id, off] : prog->uploads) uploaded[id] = 1;
    if (upl_bytes || !prog->dims_host.empty()) {
      auto mem = std::make_unique<DevMem>();
      if (int rc = mem->alloc(upl_bytes + 8 * prog->dims_host.size() + 16)) return rc;
      prog->upl_dev = mem->p;
      prog->dims_dev = reinterpret_cast<int64_t*>(static_cast<char*>(mem->p) + ((upl_bytes + 15) & ~(size_t)15));
      for (auto [id, off] : prog->uploads) prog->slots[id].ptr = static_cast<char*>(mem->p) + off;
      prog->mems.push_back(std::move(mem));
    }
    for (size_t i = 0; i < prog->slots.size(); ++i) {
      Slot& s = prog->slots[i];
      if (uploaded[i]) continue;
      if (s.kind == Slot::kInput && free_rule_[s.io] == 1) {  // only its shape is read
        s.ptr = nullptr;
        continue;
      }
      const bool staged = (s.kind == Slot::kInput && (!in[s.io].on_device || free_rule_[s.io] == 2)) ||
                          (s.kind == Slot::kOutput && !out[s.io].on_device);
      if (s.kind != Slot::kTemp && !staged) continue;
      const size_t bytes = (size_t)std::max<int64_t>(numel_of(s.shape), 1) * std::max(dtype_size(s.dtype), 1);
      if (staged || s.dtype == kU8 || last[i] < 0) {
        auto mem = std::make_unique<DevMem>();
        if (int rc = mem->alloc(bytes)) return rc;
        if (s.dtype == kU8) cudaMemset(mem->p, 0, bytes);  // attention workspaces start zeroed
        s.ptr = mem->p;
        prog->mems.push_back(std::move(mem));
      } else {
        arena.push_back(Place{(int)i, (bytes + 255) & ~(size_t)255, 0});
      }
    }
    // largest first; each at the lowest offset clear of every placed buffer whose lifetime overlaps
    std::sort(arena.begin(), arena.end(), [](const Place& a, const Place& b) {
      return a.bytes != b.bytes ? a.bytes > b.bytes : a.id < b.id;
    });
    size_t arena_bytes = 0;
    for (size_t a = 0; a < arena.size(); ++a) {
      std::vector<std::pair<size_t, size_t>> busy;
      for (size_t b = 0; b < a; ++b)
        if (first[arena[b].id] <= last[arena[a].id] && first[arena[a].id] <= last[arena[b].id])
          busy.push_back({arena[b].off, arena[b].off + arena[b].bytes});
      std::sort(busy.begin(), busy.end());
      size_t off = 0;
      for (auto [lo, hi] : busy) {
        if (off + arena[a].bytes <= lo) break;
        off = std::max(off, hi);
      }
      arena[a].off = off;
      arena_bytes = std::max(arena_bytes, off + arena[a].bytes);
    }
    if (!arena.empty()) {
      auto mem = std::make_unique<DevMem>();
      if (int rc = mem->alloc(arena_bytes)) return rc;
      for (const Place& pl : arena) prog->slots[pl.id].ptr = static_cast<char*>(mem->p) + pl.off;
      prog->mems.push_back(std::move(mem));
    }
    for (const Step& stp : steps_)
      if (stp.kind == StepKind::kGqa) {
        const int rows = (int)prog->slots[stp.in[0]].shape[1];
        prog->path = rows > 1 ? 1 : (prog->path == 1 ? 1 : 0);
      }
    it = programs_.emplace(key, std::move(prog)).first;
  }
  Program& prog = *it->second;
  std::vector<Slot>& S = prog.slots;
  // bind boundary tensors
  std::string ptr_key;
  for (auto& s : S) {
    if (s.kind == Slot::kInput && free_rule_[s.io]) {
      // copied in by stage_dynamic (key-axis inputs) or never read (shape-only inputs)
    } else if (s.kind == Slot::kInput) {
      const TensorArg& a = in[s.io];
      if (a.on_device) {
        s.ptr = a.data;
      } else {
        const size_t bytes = (size_t)numel_of(s.shape) * dtype_size(s.dtype);
        if (bytes) B200EP_CUDA_RET(cudaMemcpyAsync(s.ptr, a.data, bytes, cudaMemcpyHostToDevice, st));
        if (!s.host_copy.empty()) memcpy(s.host_copy.data(), a.data, s.host_copy.size());
        if (sum) {
          std::lock_guard<std::mutex> sl(sum->mu);
          sum->h2d_bytes += (int64_t)bytes;
        }
      }
    } else if (s.kind == Slot::kOutput && out[s.io].on_device) {
      s.ptr = out[s.io].data;
    }
    if (s.kind == Slot::kInput || s.kind == Slot::kOutput) {
      char buf[32];
      snprintf(buf, sizeof buf, "%p;", s.ptr);
      ptr_key += buf;
    }
  }
  if (int rc = stage_dynamic(prog, in, st)) return rc;
  ++stats_.runs;
  const bool use_graph = cfg_.cuda_graph && !env_on("ONNXRUNTIME_EP_B200_NO_GRAPH");
  const int64_t replays0 = stats_.graph_replays, captures0 = stats_.graph_captures;
  if (use_graph) {
    auto g = prog.graphs.find(ptr_key);
    if (g == prog.graphs.end()) {
      // The first run of a key executes eagerly (it also initialises lazily configured kernel
      // attributes); the second captures.
      if (prog.graphs.count("#warm" + ptr_key) == 0) {
        prog.graphs["#warm" + ptr_key] = nullptr;
        if (int rc = launch_steps(S, prog, st)) return rc;
      } else {
        cudaStreamCaptureStatus cs;
        B200EP_CUDA_RET(cudaStreamIsCapturing(st, &cs));
        if (cs != cudaStreamCaptureStatusNone) {
          if (int rc = launch_steps(S, prog, st)) return rc;
        } else {
          cudaGraph_t graph = nullptr;
          B200EP_CUDA_RET(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
          int rc = launch_steps(S, prog, st);
          cudaError_t ce = cudaStreamEndCapture(st, &graph);
          if (rc) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
          }
          B200EP_CUDA_RET(ce);
          cudaGraphExec_t exec = nullptr;
          ce = cudaGraphInstantiate(&exec, graph, 0);
          cudaGraphDestroy(graph);
          B200EP_CUDA_RET(ce);
          prog.graphs[ptr_key] = exec;
          ++stats_.graph_captures;
          B200EP_CUDA_RET(cudaGraphLaunch(exec, st));
          ++stats_.graph_replays;
        }
      }
    } else {
      B200EP_CUDA_RET(cudaGraphLaunch(g->second, st));
      ++stats_.graph_replays;
    }
    auto g2 = prog.graphs.find(ptr_key);
    if (g2 != prog.graphs.end() && g2->second) {
      last_sig_ = std::move(sig);
      last_prog_ = &prog;
      last_exec_ = g2->second;
    }
  } else {
    if (int rc = launch_steps(S, prog, st)) return rc;
  }
  // host outputs
  int64_t d2h = 0;
  for (auto& s : S)
    if (s.kind == Slot::kOutput && !out[s.io].on_device) {
      const size_t bytes = (size_t)numel_of(s.shape) * dtype_size(s.dtype);
      if (bytes) B200EP_CUDA_RET(cudaMemcpyAsync(out[s.io].data, s.ptr, bytes, cudaMemcpyDeviceToHost, st));
      d2h += (int64_t)bytes;
    }
  if (sum) {
    std::lock_guard<std::mutex> sl(sum->mu);
    ++(prog.path == 0 ? sum->path_decode : prog.path == 1 ? sum->path_prefill : sum->path_general);
    const int64_t rp = stats_.graph_replays - replays0, cp = stats_.graph_captures - captures0;
    sum->graph_replays += rp;
    sum->graph_captures += cp;
    if (!rp) ++sum->eager_runs;
    sum->d2h_bytes += d2h;
  }
  bool any_host_out = false;
  for (auto& o : out) any_host_out |= !o.on_device;
  if (any_host_out) B200EP_CUDA_RET(cudaStreamSynchronize(st));
  return B200EP_OK;
}

std::string Plan::preview() const {
  auto fnv = [](const std::vector<uint8_t>& b) {
    uint64_t h = 1469598103934665603ull;
    for (uint8_t c : b) h = (h ^ c) * 1099511628211ull;
    return h;
  };
  std::ostringstream o;
  o << "[";
  for (size_t i = 0; i < steps_.size(); ++i) {
    const Step& st = steps_[i];
    o << (i ? "," : "") << "{\"op\":\"" << step_kind_name(st.kind) << "\",\"name\":\"" << st.name << "\"";
    if (st.kind == StepKind::kMnb) {
      o << ",\"N\":" << st.N << ",\"K\":" << st.K;
      const char* keys[3] = {"B", "scales", "zp"};
      const int ids[3] = {st.wB, st.wS, st.wZ};
      for (int j = 0; j < 3; ++j) {
        auto it = pending_consts_.find(ids[j]);
        if (ids[j] >= 0 && it != pending_consts_.end())
          o << ",\"" << keys[j] << "\":\"" << std::hex << fnv(it->second->bytes) << std::dec << "\"";
      }
    } else if (st.kind == StepKind::kGqa) {
      o << ",\"heads\":" << st.num_heads << ",\"kv_heads\":" << st.kv_heads;
    } else if (st.kind == StepKind::kSiluMul || st.kind == StepKind::kAllGather) {
      o << ",\"N\":" << st.N;
    }
    o << "}";
  }
  o << "]";
  return o.str();
}

std::string Plan::describe() const {
  std::ostringstream o;
  o << "{\"nodes\":" << stats_.nodes << ",\"steps\":" << steps_.size() << ",\"fused_qkv\":" << stats_.fused_qkv
    << ",\"fused_swiglu\":" << stats_.fused_swiglu << ",\"fused_norm\":" << stats_.fused_norm
    << ",\"fused_act\":" << stats_.fused_act << ",\"swiglu_epilogue\":" << stats_.swiglu_epilogue
    << ",\"peer_allreduce\":" << stats_.peer_allreduce
    << ",\"weight_bytes\":" << stats_.weight_bytes
    << ",\"runs\":" << stats_.runs << ",\"graph_captures\":" << stats_.graph_captures
    << ",\"graph_replays\":" << stats_.graph_replays;
  int npk = 0;
  for (auto& st : steps_) npk += st.prepacked;
  o << ",\"prepacked_matmulnbits\":" << npk << ",\"ops\":[";
  for (size_t i = 0; i < steps_.size(); ++i) o << (i ? "," : "") << "\"" << step_kind_name(steps_[i].kind) << "\"";
  o << "]}";
  return o.str();
}

}  // namespace b200ep
