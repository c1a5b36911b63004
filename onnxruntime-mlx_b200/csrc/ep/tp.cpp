// Tensor parallelism over NCCL (one process per GPU).  The plan shards column-parallel projections
// (q/k/v, gate/up: output rows split), row-parallel projections (o, down: K split at block
// boundaries, followed by an all-reduce of the partial sums) and attention by KV head; the
// vocabulary-split lm_head is followed by an all-gather.  Collectives are issued on the plan's
// stream and are captured into its CUDA graph like the kernels.
#include "tp.h"

#include <cstring>
#include <string>

#include "../common.cuh"
#include "plan.h"

#ifdef B200EP_HAVE_NCCL
#include <nccl.h>
#endif

namespace b200ep {

TpContext::~TpContext() {
#ifdef B200EP_HAVE_NCCL
  if (owns_comm && comm) ncclCommDestroy(static_cast<ncclComm_t>(comm));
#endif
}

int tp_collective(const TpContext& tp, const Step& s, const std::vector<Slot>& S, cudaStream_t st) {
#ifdef B200EP_HAVE_NCCL
  const Slot& x = S[s.in[0]];
  const Slot& y = S[s.out[0]];
  ncclDataType_t dt = x.dtype == kF16 ? ncclFloat16 : x.dtype == kBF16 ? ncclBfloat16 : ncclFloat32;
  ncclResult_t r;
  if (s.kind == StepKind::kAllReduce) {
    r = ncclAllReduce(x.ptr, y.ptr, (size_t)x.numel(), dt, ncclSum, static_cast<ncclComm_t>(tp.comm), st);
  } else {
    // gather [rows, shard] blocks from every rank into [world, rows, shard]; the plan's gather
    // step owns a staging slot laid out rank-major and permutes it to [rows, world*shard]
    r = ncclAllGather(x.ptr, y.ptr, (size_t)x.numel(), dt, static_cast<ncclComm_t>(tp.comm), st);
  }
  if (r != ncclSuccess) return set_error(B200EP_ENCCL, std::string("NCCL: ") + ncclGetErrorString(r));
  return B200EP_OK;
#else
  (void)tp;
  (void)s;
  (void)S;
  (void)st;
  return set_error(B200EP_EUNSUPPORTED, "library built without NCCL");
#endif
}

}  // namespace b200ep
