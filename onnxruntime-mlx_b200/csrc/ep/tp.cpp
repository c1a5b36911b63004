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
    // every rank holds [rows, shard] columns of [rows, shard * world]: gather rank-major, then
    // place each rank's block at its column offset (one 2-D copy per rank; none for one row)
    const int64_t shard = s.shard_cols, rows = x.numel() / std::max<int64_t>(shard, 1);
    if (rows == 1) {
      r = ncclAllGather(x.ptr, y.ptr, (size_t)x.numel(), dt, static_cast<ncclComm_t>(tp.comm), st);
    } else {
      const Slot& stage = S[s.ws_slot];
      r = ncclAllGather(x.ptr, stage.ptr, (size_t)x.numel(), dt, static_cast<ncclComm_t>(tp.comm), st);
      const size_t esz = (size_t)dtype_size(x.dtype);
      for (int k = 0; r == ncclSuccess && k < tp.world; ++k) {
        cudaError_t e = cudaMemcpy2DAsync(static_cast<char*>(y.ptr) + k * shard * esz, (size_t)s.N * esz,
                                          static_cast<const char*>(stage.ptr) + (size_t)k * rows * shard * esz,
                                          shard * esz, shard * esz, rows, cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return cuda_status(e, "tensor-parallel gather placement");
      }
    }
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
